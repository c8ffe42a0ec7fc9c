"""Multi-GPU runners on one box (one process per GPU, torchrun-launched).

Data-parallel replicas reduce gradients with the fused cross-replica kernel
(K1) over NVLink peer memory, overlapped with backward bucket by bucket; the
optional fault-tolerance Manager takes a quorum every step and votes on the
commit (the SHIFT step of shift_full/train.py:506-627).  Each replica
processes its share of the fixed global batch.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..engine import Engine, synthetic_batch
from ..graphs import StepGraphs, graphs_enabled
from ..models.qwen_moe import MoEConfig
from ..ops._ext import check_status, ext
from .symmetric import CrossReplicaFused, SymmetricHeap, _tag


def _order(layer: int, layers: int) -> int:
    if layer == -1:
        return 0
    if layer == -2:
        return layers + 1
    return layers - layer


class ReplicaDPRunner:
    """R replicas x 1 GPU; rank r is replica r."""

    def __init__(self, cfg: MoEConfig, n_gpus: int, rank: int, local_rank: int, batch: int, seq: int,
                 with_manager: bool = False):
        if batch % n_gpus:
            raise ValueError(f"global batch {batch} is not divisible by {n_gpus} replicas")
        self.layout = f"dp{n_gpus} (replicas x 1 GPU, fused NVLink reduce+AdamW)"
        self.cfg = cfg
        self.rank, self.world = rank, n_gpus
        self.device = torch.device("cuda", local_rank)
        self.B, self.S = batch // n_gpus, seq
        self.engine = Engine(cfg, self.device)
        store = dist.distributed_c10d._get_default_store()
        self.heap = SymmetricHeap(store, f"r{rank}", self.device)
        self.fused = CrossReplicaFused(self.engine, self.heap)
        self.fused.nccl_group = dist.group.WORLD       # the K1 baseline arm (SHIFT_K1=nccl) reduces over it
        dist.barrier()
        self.fused.configure([f"r{i}" for i in range(n_gpus)])
        layers = cfg.layers
        self.engine.model.layer_done_hook = lambda layer: self.fused.on_layer_done(_order(layer, layers))
        sl = slice(rank * self.B, (rank + 1) * self.B)
        self.dev_batches = [synthetic_batch(cfg, i, batch, seq)[sl].to(self.device) for i in range(4)]
        self.host = synthetic_batch(cfg, 10_000, batch, seq)[sl].contiguous().pin_memory()
        self.tokens = torch.empty(self.B, seq + 1, dtype=torch.int32, device=self.device)
        self.graphs = StepGraphs(self.device, graphs_enabled())
        self.manager = None
        self.step_no = 0
        self.eager_until = 2
        if with_manager:
            self._init_manager(store)
        dist.barrier()

    def _init_manager(self, store):
        from ..ft.manager import Manager
        from ..ft.native import LighthouseServer
        if self.rank == 0:
            self._lh = LighthouseServer("127.0.0.1:0", min_replicas=self.world, join_timeout_ms=500,
                                        heartbeat_timeout_ms=2000, quorum_tick_ms=20)
            store.set("bench/lighthouse", self._lh.address)
        addr = store.get("bench/lighthouse").decode()
        # every replica must take part in every step of the benchmark
        self.manager = Manager(None, None, None, self.world, f"shift{self.rank}", addr, rank=0, world_size=1,
                               store=store, local_prefix=f"/bench{self.rank}")

    def _device_step(self):
        step = self.step_no
        tok, lab = self.tokens[:, :-1], self.tokens[:, 1:]
        self.engine.nonfinite.zero_()
        self.fused.begin_step(step, prepare=False)
        loss = self.engine.forward_backward([(tok, lab)], self.B, self.S)
        self.fused.finish_step()
        return loss

    def _train(self):
        if self.manager is not None:
            self.manager.start_quorum()
        step = self.step_no
        self.engine.prepare_step(_tag(step))
        if step < self.eager_until:      # eager warm-up steps; buffer-reuse waits start at step 2
            loss = self._device_step()
        else:
            loss = self.graphs.run((self.engine.store.cur, step % 2), self._device_step)
        commit = True
        if self.manager is not None:
            commit = self.manager.should_commit()
        if commit:
            self.engine.commit()
        self.step_no += 1
        return loss

    def step(self, i: int):
        self.tokens.copy_(self.dev_batches[i % len(self.dev_batches)])
        return self._train()

    def set_k1_mode(self, mode: str):
        """Switch the cross-replica reduction between the fused peer-memory
        kernels ("auto") and the NCCL baseline ("nccl"); the step graphs are
        captured again after two eager steps."""
        torch.cuda.synchronize()
        self.graphs.reset()
        self.fused.mode = mode
        self.eager_until = self.step_no + 2

    # ------------------------------------------------------------------ correctness checks
    def initial_full_state(self) -> dict:
        """Whole-model weights of this replica (call before training): every
        replica starts from the same seeded initialisation."""
        return {n: t.clone() for n, t in self.engine.store.model_state_dict().items()}

    def state_fingerprints(self) -> dict:
        return state_fingerprints(self.engine.store, replica=self.rank, position="dp")

    def step_e2e(self, i: int):
        self.tokens.copy_(self.host, non_blocking=True)
        loss = self._train()
        val = loss.item()
        return val, self.host.numel() * self.host.element_size(), 4

    def close(self):
        torch.cuda.synchronize()
        self.graphs.reset()
        check_status(self.device)
        if self.manager is not None:
            self.manager.shutdown()
        dist.barrier()
        self.heap.close_peers()


def state_fingerprints(store, replica: int, position: str) -> dict:
    """64-bit fingerprints of this rank's committed flat state (bf16 params,
    fp32 master, Adam moments): replicas of one position must agree bit for
    bit after every committed step."""
    fp = ext().fingerprint
    c = store.cur
    return {"replica": replica, "position": position, "param": fp(store.param[c]), "master": fp(store.master[c]),
            "exp_avg": fp(store.exp_avg[c]), "exp_avg_sq": fp(store.exp_avg_sq[c]), "step": store.step}


def make_parallel_runner(n_gpus: int, rank: int, local_rank: int, batch: int, seq: int, cfg: MoEConfig):
    """Default layouts: 2 GPUs -> 2 replicas x 1; 4 -> 2 replicas x TP2;
    8 -> 2 replicas x (TP2 x PP2).  SHIFT_LAYOUT=dp|tp|tppp overrides."""
    layout = os.environ.get("SHIFT_LAYOUT") or {2: "dp", 4: "tp", 8: "tppp"}.get(n_gpus, "dp")
    if layout == "dp":
        return ReplicaDPRunner(cfg, n_gpus, rank, local_rank, batch, seq,
                               with_manager=os.environ.get("SHIFT_BENCH_FT", "1") == "1")
    from .tp_pp import make_model_parallel_runner
    return make_model_parallel_runner(layout, cfg, n_gpus, rank, local_rank, batch, seq)
