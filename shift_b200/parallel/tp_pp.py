"""Replicas of TP x PP GPUs on one box (the 2 replicas x 4 GPU layout).

Global rank = replica * (tp*pp) + stage * tp + tp_rank.  Inside a replica:
tensor parallelism with sequence parallelism and experts split over the TP
pair (``parallel.tp``), pipeline parallelism with a 1F1B schedule over
microbatches of two sequences; activations and gradients travel through
peer-memory slots written by a copy kernel and guarded by step-tag flags
(``parallel.pipe.PipePeer``, capturable in the step's CUDA graph), or on NCCL
p2p as the baseline (``SHIFT_PP_BACKEND=nccl``; the reference keeps PP on NCCL
p2p, shift_full/train.py:552).  Across replicas: the fused peer-memory
reduce + AdamW (K1) per bucket, overlapped with the last microbatch's
backward; TP-replicated parameters are summed over the TP pair and averaged
over replicas inside the same kernel.
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..engine import Engine, synthetic_batch
from ..models.qwen_moe import TP_SHARDED, MoEConfig, Partition, param_specs
from ..ops._ext import check_status
from ..graphs import StepGraphs, graphs_enabled
from .replicas import _order, state_fingerprints
from .symmetric import CrossReplicaFused, SymmetricHeap, _tag
from .assemble import initial_model_parallel_weights, shard_seed
from .pipe import ACT, GRAD, PipeNccl, PipePeer
from .tp import TPComm, TPPeer


def _is_sharded(name: str) -> bool:
    return any(name.endswith(s) for s in TP_SHARDED)


class ModelParallelRunner:
    def __init__(self, cfg: MoEConfig, n_gpus: int, rank: int, local_rank: int, batch: int, seq: int,
                 replicas: int, tp: int, pp: int, microbatch: int | None = None, tp_backend: str | None = None,
                 pp_backend: str | None = None, with_manager: bool | None = None):
        if microbatch is None:
            # one microbatch per replica without pipelining; with it, two sequences per
            # microbatch.  At 2 replicas x (TP2 x PP2) on B200 one sequence per
            # microbatch (four microbatches, a 1F1B bubble of 1/5) measured 19.9 ms
            # per step against 15.4 ms for two (bubble 1/3): a TP rank's 1,024-row
            # GEMMs and single-sequence attention leave most SMs idle, which costs
            # more than the larger bubble
            microbatch = batch // replicas if pp == 1 else min(2, batch // replicas)
        if replicas * tp * pp != n_gpus:
            raise ValueError(f"{replicas} x tp{tp} x pp{pp} != {n_gpus} GPUs")
        if batch % (replicas * microbatch):
            raise ValueError("global batch must split evenly over replicas and microbatches")
        if cfg.layers % pp or cfg.experts % tp or cfg.heads % tp or cfg.kv_heads % tp:
            raise ValueError("layers / experts / heads must divide by pp / tp")
        self.layout = f"{replicas}x(tp{tp},pp{pp}) sp+ep-over-tp, 1F1B, fused NVLink reduce+AdamW"
        self.cfg, self.rank = cfg, rank
        per = tp * pp
        self.r, rem = divmod(rank, per)
        self.s, self.t = divmod(rem, tp)
        self.R, self.TP, self.PP = replicas, tp, pp
        self.device = torch.device("cuda", local_rank)
        self.S = seq
        self.mb = microbatch
        self.M = batch // replicas // microbatch
        # ---- process groups (every rank creates every group, in the same order) ----
        self.tp_group = None
        for r in range(replicas):
            for s in range(pp):
                g = dist.new_group([r * per + s * tp + t for t in range(tp)])
                if r == self.r and s == self.s:
                    self.tp_group = g
        self.pp_ranks = [self.r * per + s * tp + self.t for s in range(pp)]
        self.pp_group = None
        for r in range(replicas):
            for t in range(tp):
                g = dist.new_group([r * per + s * tp + t for s in range(pp)])
                if r == self.r and t == self.t:
                    self.pp_group = g
        # ---- model partition ----
        lps = cfg.layers // pp
        e_per = cfg.experts // tp
        part = Partition(layer_lo=self.s * lps, layer_hi=(self.s + 1) * lps, has_embed=self.s == 0,
                         has_head=self.s == pp - 1, expert_lo=self.t * e_per, expert_hi=(self.t + 1) * e_per,
                         tp_size=tp)
        specs = param_specs(cfg, part)
        rep = [s for s in specs if not _is_sharded(s.name)]
        shard = [s for s in specs if _is_sharded(s.name)]
        t_rank = self.t

        def seed_of(spec):
            return shard_seed(spec.name, t_rank)

        store = dist.distributed_c10d._get_default_store()
        self.heap = SymmetricHeap(store, f"r{self.r}s{self.s}t{self.t}", self.device)
        self.tp_backend = tp_backend or os.environ.get("SHIFT_TP_BACKEND", "peer")
        if self.tp_backend == "peer" and tp == 2:
            # activations cross the TP pair inside our kernels (symmetric memory)
            self.comm = TPPeer(self.tp_group, self.t, tp, self.device, self.heap, f"r{self.r}s{self.s}t{1 - self.t}",
                               tokens=microbatch * seq, hidden=cfg.hidden, layers=range(part.layer_lo, part.layer_hi),
                               microbatches=self.M)
        else:
            self.tp_backend = "nccl"
            self.comm = TPComm(self.tp_group, self.t, tp, self.device)
        self.layout += f", TP over {'peer memory (fused kernels)' if self.tp_backend == 'peer' else 'NCCL'}"
        self.engine = Engine(cfg, self.device, part=part, specs=rep + shard, seed_of=seed_of, tp=self.comm)
        st = self.engine.store
        self.rep_end = st.offsets[shard[0].name][0] if shard else st.numel
        # ---- fused cross-replica (and cross-TP for replicated params) reduction ----
        self.fused = CrossReplicaFused(self.engine, self.heap)
        if self.fused.mode == "nccl":
            raise ValueError("the NCCL K1 baseline (SHIFT_K1=nccl) is wired for the replicas x 1 GPU layout only")
        dist.barrier()
        if isinstance(self.comm, TPPeer):
            self.comm.connect(self.engine.step_block.dev)
        rep_src = [f"r{r}s{self.s}t{t}" for r in range(replicas) for t in range(tp)]
        shard_src = [f"r{r}s{self.s}t{self.t}" for r in range(replicas)]
        owners = sorted(set(rep_src) | set(shard_src))
        self.fused.configure_segments(owners, [(0, self.rep_end, rep_src, 1.0 / replicas),
                                               (self.rep_end, st.numel, shard_src, 1.0 / replicas)])
        layers = cfg.layers
        self._hook = lambda layer: self.fused.on_layer_done(_order(layer, layers))
        # ---- data: replica r takes sequences [r*B/R, (r+1)*B/R) of the global batch ----
        b_per = batch // replicas
        sl = slice(self.r * b_per, (self.r + 1) * b_per)
        self.dev_batches = [synthetic_batch(cfg, i, batch, seq)[sl].to(self.device) for i in range(2)]
        self.host = synthetic_batch(cfg, 10_000, batch, seq)[sl].contiguous().pin_memory()
        self.tokens = torch.empty_like(self.dev_batches[0])      # static step input (graph replay)
        use_graphs = graphs_enabled()
        if self.tp_backend == "nccl" and tp > 1:
            use_graphs = use_graphs and os.environ.get("SHIFT_PP_GRAPHS") == "1"
        self.tok_loc = self.mb * seq // tp
        # ---- pipeline send/recv: peer memory (default) or the NCCL baseline ----
        self.pipe = None
        if pp > 1:
            self.pp_backend = pp_backend or os.environ.get("SHIFT_PP_BACKEND", "peer")
            act_shape, grad_shape = (2, self.tok_loc, cfg.hidden), (self.tok_loc, cfg.hidden)
            if self.pp_backend == "peer":
                self.pipe = PipePeer(self.heap, [f"r{self.r}s{q}t{self.t}" for q in range(pp)], self.s, act_shape,
                                     grad_shape, self.M, self.device, self.engine.step_block.dev)
            else:
                self.pp_backend = "nccl"
                self.pipe = PipeNccl(self.pp_group, self.pp_ranks, self.s, act_shape, grad_shape, self.M,
                                     self.device)
            self.layout += f", PP send/recv over {'peer memory' if self.pp_backend == 'peer' else 'NCCL'}"
            use_graphs = graphs_enabled() and (self.pipe.graphable or os.environ.get("SHIFT_PP_GRAPHS") == "1")
            if self.tp_backend == "nccl" and tp > 1:
                use_graphs = use_graphs and os.environ.get("SHIFT_PP_GRAPHS") == "1"
        self.graphs = StepGraphs(self.device, use_graphs)
        self.step_no = 0
        dist.barrier()
        if isinstance(self.pipe, PipePeer):
            self.pipe.connect()
        # ---- fault tolerance: quorum + commit vote of every replica every step ----
        self.manager = None
        if with_manager is None:
            with_manager = os.environ.get("SHIFT_BENCH_FT", "1") == "1"
        if with_manager and replicas > 1:
            self._init_manager(store, per)
        dist.barrier()

    def _init_manager(self, store, per):
        from ..ft.manager import Manager
        from ..ft.native import LighthouseServer
        if self.rank == 0:
            self._lh = LighthouseServer("127.0.0.1:0", min_replicas=self.R, join_timeout_ms=500,
                                        heartbeat_timeout_ms=2000, quorum_tick_ms=20)
            store.set("bench/lighthouse", self._lh.address)
        addr = store.get("bench/lighthouse").decode()
        # one manager per rank; the replica's rank 0 serves its ranks' quorum and commit votes
        self.manager = Manager(None, None, None, self.R, f"shift{self.r}", addr, rank=self.s * self.TP + self.t,
                               world_size=per, store=store, local_prefix=f"/bench{self.r}")

    # ------------------------------------------------------------------ one step (1F1B)
    def _slot(self, i):
        if isinstance(self.comm, TPPeer):
            self.comm.set_slot(i, self.step_no % 2)

    def _fwd(self, i, data, hidden):
        self._slot(i)
        model = self.engine.model
        tok = data[i * self.mb:(i + 1) * self.mb]
        out, loss = model.forward(tok[:, :-1] if self.s == 0 else None,
                                  None if self.s == 0 else (hidden[0], hidden[1]),
                                  tok[:, 1:] if self.s == self.PP - 1 else None, self.mb, self.S,
                                  loss_scale=1.0 / (self.M * self.mb * self.S))
        if loss is not None:
            self._loss = loss if self._loss is None else self._loss + loss
        return None if out is None else torch.stack([out[0], out[1]])

    def _bwd(self, i, dout):
        self._slot(i)
        model = self.engine.model
        model._accumulate = i > 0
        model._last_microbatch = i == self.M - 1
        model.layer_done_hook = self._hook if i == self.M - 1 else None
        d = model.backward(dout)        # the same gradient reaches both halves of the stage input pair
        model.layer_done_hook = None
        return d

    def _train(self, data):
        """One step.  Without pipelining (no NCCL on the step's path when the
        TP pair runs over peer memory) the step is captured as a CUDA graph per
        (state generation, step parity) after two eager steps; with pipelining
        it runs eagerly unless SHIFT_PP_GRAPHS=1 (NCCL p2p inside the graph)."""
        if self.manager is not None:
            self.manager.start_quorum()
        step = self.step_no
        self.engine.prepare_step(_tag(step))
        if data is not self.tokens:
            self.tokens.copy_(data, non_blocking=True)
        if step < 2 or not self.graphs.enabled:
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

    def _device_step(self):
        data = self.tokens
        eng = self.engine
        eng.nonfinite.zero_()
        self.fused.begin_step(self.step_no, prepare=False)
        eng.store.zero_grad()
        self._loss = None
        M, s, pp = self.M, self.s, self.PP
        first, last = s == 0, s == pp - 1
        pipe = self.pipe
        if pipe is not None:
            pipe.set_parity(self.step_no % 2)
        # Weight gradients off the pipeline's critical path: the last stage
        # queues every microbatch's weight-gradient GEMMs until its last input
        # gradient has been sent, so the stage below gets its gradients a
        # weight-gradient pass earlier; the other stages run them right after
        # each backward, in the time they would wait for the next gradient
        # (at PP2 with two microbatches the step takes 7 backward-pass units
        # instead of 9 -- the first bubble-filling split of Qi et al.'s
        # zero-bubble pipeline schedules): measured 30.3 -> 25.7 ms per step
        # at PP2 on two B200s.  SHIFT_PP_DEFER_WGRAD=0 turns it off
        defer = pipe is not None and os.environ.get("SHIFT_PP_DEFER_WGRAD", "1") == "1"
        eng.model.defer_wgrad = defer
        n_warm = min(pp - s - 1, M)
        n_rem = M - n_warm
        for i in range(n_warm):
            x = None if first else pipe.exchange(recv=(ACT, i))
            y = self._fwd(i, data, x)
            pipe.exchange(send=(ACT, i, y))
        x = None if (first or n_rem == 0) else pipe.exchange(recv=(ACT, n_warm))
        for j in range(n_rem):
            i = n_warm + j
            y = self._fwd(i, data, x)
            dy = None if last else pipe.exchange(send=(ACT, i, y), recv=(GRAD, j))
            dx = self._bwd(j, dy)
            if j == n_rem - 1:
                if not first:
                    pipe.exchange(send=(GRAD, j, dx))
                if defer and not last:
                    eng.model.flush_wgrad()
            else:
                if defer and first:
                    eng.model.flush_wgrad()
                x = None if first else pipe.exchange(send=(GRAD, j, dx), recv=(ACT, i + 1))
                if defer and not first and not last:
                    eng.model.flush_wgrad()
        for j in range(n_rem, M):
            dy = None if last else pipe.exchange(recv=(GRAD, j))
            dx = self._bwd(j, dy)
            if not first:
                pipe.exchange(send=(GRAD, j, dx))
            if defer and not last:
                eng.model.flush_wgrad()
        if defer:
            eng.model.flush_wgrad()
            eng.model.defer_wgrad = False
        eng.model._accumulate = False
        self.fused.finish_step()
        if self._loss is None:
            return torch.zeros((), device=self.device)
        # the model returns token sums; this rank's share of the replica's mean loss
        return self._loss / float(self.M * self.mb * self.S)

    def step(self, i: int):
        return self._train(self.dev_batches[i % len(self.dev_batches)])

    # ------------------------------------------------------------------ correctness checks
    def initial_full_state(self) -> dict:
        """Whole-model initial weights of a replica, rebuilt on the host from
        the per-shard seeds (no shard moves)."""
        return initial_model_parallel_weights(self.cfg, self.TP, self.PP)

    def state_fingerprints(self) -> dict:
        return state_fingerprints(self.engine.store, replica=self.r, position=f"s{self.s}t{self.t}")

    def step_e2e(self, i: int):
        loss = self._train(self.host)
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


def make_model_parallel_runner(layout: str, cfg, n_gpus, rank, local_rank, batch, seq):
    """layout: 'tp' (replicas x TP2), 'tppp' (replicas x TP2 x PP2), 'pp'
    (replicas x PP2, no tensor parallelism) or 'auto'."""
    if layout == "auto":
        layout = {4: "tp", 8: "tppp"}.get(n_gpus, "tp")
    tp = 1 if layout == "pp" else 2
    pp = 2 if layout in ("tppp", "pp") else 1
    replicas = n_gpus // (tp * pp)
    mb = os.environ.get("SHIFT_MICROBATCH")      # sequences per pipeline microbatch
    return ModelParallelRunner(cfg, n_gpus, rank, local_rank, batch, seq, replicas, tp, pp,
                               microbatch=int(mb) if mb else None)
