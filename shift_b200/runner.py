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

import os

import torch

from .engine import Engine, synthetic_batch
from .graphs import StepGraphs, graphs_enabled
from .models.qwen_moe import MoEConfig
from .parallel.symmetric import _tag


class SingleRunner:
    layout = "dp1"

    def __init__(self, cfg: MoEConfig, device, batch: int, seq: int, n_prefetch: int = 4,
                 graphs: bool | None = None, overlap_optimizer: bool | None = None):
        self.cfg = cfg
        self.engine = Engine(cfg, device)
        self.B, self.S = batch, seq
        self.device = torch.device(device)
        # optional: AdamW per gradient bucket on a side stream as soon as
        # backward has written the bucket (the cross-replica step's machinery
        # with this GPU as the only member).  Off by default: on one GPU the
        # memory-bound updates slow the memory-bound parts of backward about
        # as much as they save at the end (measured 36.85 ms vs 36.00 ms per
        # step with one full-model pass after backward)
        if overlap_optimizer is None:
            overlap_optimizer = os.environ.get("SHIFT_N1_OVERLAP", "0") == "1"
        self.fused = None
        if overlap_optimizer and self.device.type == "cuda":
            from .parallel.replicas import _order
            from .parallel.symmetric import CrossReplicaFused, SymmetricHeap
            self.heap = SymmetricHeap(None, "solo", self.device)
            self.fused = CrossReplicaFused(self.engine, self.heap, mode="one")
            self.fused.configure(["solo"])
            layers = cfg.layers
            self.engine.model.layer_done_hook = lambda layer: self.fused.on_layer_done(_order(layer, layers))
            self.layout = "dp1 (AdamW per bucket overlapped with backward)"
        # device-resident inputs for the kernel-timed loop
        self.dev_batches = [synthetic_batch(cfg, i, batch, seq).to(self.device) for i in range(n_prefetch)]
        self.host = synthetic_batch(cfg, 10_000, batch, seq).pin_memory()
        # the step reads its tokens from this buffer (static for graph replay)
        self.tokens = torch.empty(batch, seq + 1, dtype=torch.int32, device=self.device)
        self.graphs = StepGraphs(self.device, graphs_enabled() if graphs is None else graphs)
        self.step_no = 0

    def _device_step(self):
        tok, lab = self.tokens[:, :-1], self.tokens[:, 1:]
        if self.fused is not None:
            self.engine.nonfinite.zero_()
            self.fused.begin_step(self.step_no, prepare=False)
            loss = self.engine.forward_backward([(tok, lab)], self.B, self.S)
            self.fused.finish_step()
            return loss
        loss = self.engine.forward_backward([(tok, lab)], self.B, self.S)
        self.engine.optimizer_step(prepared=True)
        return loss

    def _train(self):
        self.engine.prepare_step(_tag(self.step_no))
        if self.step_no < 2:      # eager warm-up steps (lazy initialisation)
            loss = self._device_step()
        else:
            loss = self.graphs.run(self.engine.store.cur, self._device_step)
        self.engine.commit()
        self.step_no += 1
        return loss

    def step(self, i: int):
        self.tokens.copy_(self.dev_batches[i % len(self.dev_batches)])
        return self._train()

    def step_e2e(self, i: int):
        self.tokens.copy_(self.host, non_blocking=True)
        loss = self._train()
        val = loss.item()
        return val, self.host.numel() * self.host.element_size(), 4

    def close(self):
        self.graphs.reset()


def make_runner(n_gpus: int, rank: int, local_rank: int, batch: int, seq: int, cfg: MoEConfig | None = None):
    cfg = cfg or MoEConfig.bench()
    dev = torch.device("cuda", local_rank)
    if n_gpus == 1:
        return SingleRunner(cfg, dev, batch, seq)
    from .parallel.replicas import make_parallel_runner
    return make_parallel_runner(n_gpus, rank, local_rank, batch, seq, cfg)
