"""Benchmark / training runners for each GPU count of one box.

``make_runner(n_gpus, rank, local_rank, global_batch, seq)`` returns an
object with ``step(i)`` (device-resident inputs), ``step_e2e(i)`` (pinned
host inputs copied in, loss read back) and ``layout``.

    1 GPU : one replica, whole model                      ("dp1")
    2 GPUs: 2 replicas x 1 GPU, fused cross-replica reduce + AdamW over
            NVLink peer memory                             ("2x(dp1)")
    4 GPUs: 2 replicas x TP2                                ("2x(tp2)")
    8 GPUs: 2 replicas x TP2 x PP2                          ("2x(tp2,pp2)")
"""
from __future__ import annotations

import torch

from .engine import Engine, synthetic_batch
from .models.qwen_moe import MoEConfig


class SingleRunner:
    layout = "dp1"

    def __init__(self, cfg: MoEConfig, device, batch: int, seq: int, n_prefetch: int = 4):
        self.cfg = cfg
        self.engine = Engine(cfg, device)
        self.B, self.S = batch, seq
        self.device = torch.device(device)
        # device-resident inputs for the kernel-timed loop
        self.dev_batches = [synthetic_batch(cfg, i, batch, seq).to(self.device) for i in range(n_prefetch)]
        self.host = synthetic_batch(cfg, 10_000, batch, seq).pin_memory()

    def _train(self, data):
        tok, lab = data[:, :-1], data[:, 1:]
        loss = self.engine.forward_backward([(tok, lab)], self.B, self.S)
        self.engine.optimizer_step()
        self.engine.commit()
        return loss

    def step(self, i: int):
        return self._train(self.dev_batches[i % len(self.dev_batches)])

    def step_e2e(self, i: int):
        data = self.host.to(self.device, non_blocking=True)
        loss = self._train(data)
        val = loss.item()
        return val, self.host.numel() * self.host.element_size(), 4

    def close(self):
        pass


def make_runner(n_gpus: int, rank: int, local_rank: int, batch: int, seq: int, cfg: MoEConfig | None = None):
    cfg = cfg or MoEConfig.bench()
    dev = torch.device("cuda", local_rank)
    if n_gpus == 1:
        return SingleRunner(cfg, dev, batch, seq)
    from .parallel.replicas import make_parallel_runner
    return make_parallel_runner(n_gpus, rank, local_rank, batch, seq, cfg)
