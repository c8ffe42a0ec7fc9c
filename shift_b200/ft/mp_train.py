"""Fault-tolerant worker for a model-parallel replica (TP x PP ranks).

    python -m shift_b200.control.launch --nproc TP*PP --module shift_b200.ft.mp_train -- \
        --session S --replica R --generation G --lighthouse HOST:PORT --tp 2 --pp 2 [trainer flags]

One DP replica is ``tp * pp`` processes: local rank ``s * tp + t`` holds
pipeline stage ``s`` and tensor-parallel rank ``t`` (sequence parallel, the
experts split over the TP pair).  Each step runs a 1F1B schedule over the
replica's microbatches (pipeline activations on point-to-point sends inside
the replica), sums the gradients of the TP-replicated parameters over the TP
pair, averages every rank's flat gradient with the same-coordinate rank of the
other replicas through its Manager (the cross-replica, fault-tolerant
reduction), votes, and commits -- the reference's SHIFT step
(shift_full/train.py:506-627) for a replica that is itself model-parallel.

Unplanned fault (one TP rank killed mid-backward): ``--inject sigkill_bwd@STEP``
with ``--inject-rank K`` makes local rank K SIGKILL itself in the middle of
the backward of STEP's last microbatch (``sigkill_step@STEP``: right after
STEP's commit, the form used on GPUs).  The launcher then stops the rest of
the replica, the survivors' quorum reconfigures and they continue alone; the
relaunched replica (possibly on other devices: the supervisor's
``restart_devices``) heals every rank from the same-coordinate rank of a live
replica and rejoins.  Host processes only; on GPUs the kill is taken between
steps (a rank leaves with none of its kernels in flight).
"""
from __future__ import annotations

import os
import signal
import time
from datetime import timedelta

import torch
import torch.distributed as dist

from ..engine import Engine, synthetic_batch
from ..models.qwen_moe import TP_SHARDED, MoEConfig, Partition, param_specs
from .manager import Manager, WorldSizeMode
from .process_group import ReconfigurableGroup
from .train import Worker, _free_port, parse_args as base_parse
from .transport import PackedTransport


def parse_args(argv=None):
    import argparse
    extra = argparse.ArgumentParser(add_help=False, allow_abbrev=False)
    extra.add_argument("--tp", type=int, default=2)
    extra.add_argument("--pp", type=int, default=2)
    extra.add_argument("--inject-rank", type=int, default=-1)
    extra.add_argument("--inject-replica", type=int, default=0)
    known, rest = extra.parse_known_args(argv)
    args = base_parse(rest)
    for k, v in vars(known).items():
        setattr(args, k, v)
    return args


def _sharded(name: str) -> bool:
    return any(name.endswith(s) for s in TP_SHARDED)


class GroupTP:
    """TP collectives over a process group that may lack reduce-scatter
    (gloo): all-gather by rank-ordered gather, reduce-scatter as a
    rank-ordered all-gather of the partials summed in rank order
    (deterministic, identical on both ranks)."""

    def __init__(self, group, rank: int, size: int):
        self.group, self.rank, self.size = group, rank, size

    def all_gather(self, x):
        parts = [torch.empty_like(x) for _ in range(self.size)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        return torch.cat(parts, 0)

    def reduce_scatter(self, x):
        n = x.shape[0] // self.size
        parts = [torch.empty_like(x) for _ in range(self.size)]
        dist.all_gather(parts, x.contiguous(), group=self.group)
        total = parts[0][self.rank * n:(self.rank + 1) * n].float()
        for p in parts[1:]:
            total = total + p[self.rank * n:(self.rank + 1) * n].float()
        return total.to(x.dtype)

    def all_reduce_(self, x):
        dist.all_reduce(x, group=self.group)
        return x

    def local_rows(self, x):
        n = x.shape[0] // self.size
        return x[self.rank * n:(self.rank + 1) * n]


class MPWorker(Worker):
    def __init__(self, args):
        super().__init__(args)
        if self.local_world != args.tp * args.pp:
            raise ValueError(f"replica has {self.local_world} ranks, expected tp*pp = {args.tp * args.pp}")
        self.s, self.t = divmod(self.rank, args.tp)

    # ------------------------------------------------------------------ replica-local groups
    def init_replica_groups(self):
        a = self.args
        backend = "nccl" if self.device.type == "cuda" else "gloo"
        kw = dict(device_id=self.device) if backend == "nccl" else {}
        dist.init_process_group(backend, rank=self.rank, world_size=self.local_world,
                                timeout=timedelta(seconds=a.communication_timeout), **kw)
        self.tp_group = self.pp_group = None
        for s in range(a.pp):
            g = dist.new_group([s * a.tp + t for t in range(a.tp)])
            if s == self.s:
                self.tp_group = g
        for t in range(a.tp):
            g = dist.new_group([s * a.tp + t for s in range(a.pp)])
            if t == self.t:
                self.pp_group = g
        self.pp_ranks = [s * a.tp + self.t for s in range(a.pp)]

    def data_replica(self) -> int:
        """Data rank of this replica in the sample index (the replica id; a
        planned spare uses the logical id of the replica it replaces)."""
        return self.args.replica

    def build_engine(self, ipc_state: bool = False):
        a = self.args
        cfg = self.cfg
        lps = cfg.layers // a.pp
        e_per = cfg.experts // a.tp
        part = Partition(layer_lo=self.s * lps, layer_hi=(self.s + 1) * lps, has_embed=self.s == 0,
                         has_head=self.s == a.pp - 1, expert_lo=self.t * e_per, expert_hi=(self.t + 1) * e_per,
                         tp_size=a.tp)
        specs = param_specs(cfg, part)
        rep = [sp for sp in specs if not _sharded(sp.name)]
        shard = [sp for sp in specs if _sharded(sp.name)]
        t_rank = self.t
        import zlib

        def seed_of(spec):
            salt = f"/tp{t_rank}" if _sharded(spec.name) else ""
            return a.seed + zlib.crc32((spec.name + salt).encode())

        self.comm = GroupTP(self.tp_group, self.t, a.tp) if a.tp > 1 else None
        self.engine = Engine(cfg, self.device, part=part, specs=rep + shard, seed_of=seed_of, tp=self.comm,
                             bucket_numel=a.bucket_size, ipc_state=ipc_state)
        st = self.engine.store
        self.rep_end = st.offsets[shard[0].name][0] if shard else st.numel

    # ------------------------------------------------------------------ pipeline
    def _send(self, x, to_stage):
        # non-blocking: a rank never waits for its peer to post the matching
        # receive while that peer waits for it (1F1B orders differ per stage)
        x = x.contiguous()
        self._pending.append((dist.isend(x, self.pp_ranks[to_stage], group=self.pp_group), x))

    def _recv(self, from_stage):
        buf = torch.empty(self.act_shape, dtype=self.engine.store.compute_dtype, device=self.device)
        dist.recv(buf, self.pp_ranks[from_stage], group=self.pp_group)
        return buf

    def one_step(self, step):
        """1F1B over the replica's microbatches; returns the loss sum (last stage) or 0."""
        a, eng = self.args, self.engine
        model = eng.model
        pp, s = a.pp, self.s
        first, last = s == 0, s == pp - 1
        M, S, mb = a.microbatches, a.seq_len, a.batch
        data = [synthetic_batch(self.cfg, step * (M * 4) + m * 4 + self.data_replica(), mb, S, a.data,
                                seed_base=100_000 + a.data_seed * 1_000_000).to(self.device) for m in range(M)]
        scale = 1.0 / (M * mb * S)
        losses = []

        def fwd(i, hidden):
            tok = data[i]
            out, loss = model.forward(tok[:, :-1] if first else None, None if first else (hidden[0], hidden[1]),
                                      tok[:, 1:] if last else None, mb, S, loss_scale=scale)
            if loss is not None:
                losses.append(loss)
            return None if out is None else torch.stack([out[0], out[1]])

        def bwd(j, dout):
            model._accumulate = j > 0
            model._last_microbatch = j == M - 1
            if j == M - 1 and self._kill_now(step):
                model.layer_done_hook = self._die
            d = model.backward(None if dout is None else dout[0])
            model.layer_done_hook = None
            return None if d is None else torch.stack([d, d])

        eng.store.zero_grad()
        self._pending = []
        n_warm = min(pp - s - 1, M)
        n_rem = M - n_warm
        for i in range(n_warm):
            x = None if first else self._recv(s - 1)
            self._send(fwd(i, x), s + 1)
        for j in range(n_rem):
            i = n_warm + j
            x = None if first else self._recv(s - 1)
            y = fwd(i, x)
            if not last:
                self._send(y, s + 1)
            dy = None if last else self._recv(s + 1)
            dx = bwd(j, dy)
            if not first:
                self._send(dx, s - 1)
        for j in range(n_rem, M):
            dy = None if last else self._recv(s + 1)
            dx = bwd(j, dy)
            if not first:
                self._send(dx, s - 1)
        model._accumulate = False
        for w, _ in self._pending:
            w.wait()
        self._pending = []
        total = sum(float(v) for v in losses) if losses else 0.0
        return total

    # ------------------------------------------------------------------ fault injection
    def _kill_now(self, step, kind_wanted: str = "sigkill_bwd") -> bool:
        kind, _, arg = self.args.inject.partition("@")
        return (kind == kind_wanted and step == int(arg) and self.rank == self.args.inject_rank
                and self.args.replica == self.args.inject_replica and self.args.generation == 0)

    def _replica_leaves(self, step) -> bool:
        """The planned between-steps SIGKILL of one rank of this replica
        happens after committing ``step``."""
        kind, _, arg = self.args.inject.partition("@")
        return (kind == "sigkill_step" and step == int(arg) and self.args.replica == self.args.inject_replica
                and self.args.generation == 0)

    def _die(self, layer):
        self.event("injected_sigkill", step=self.progress["updates"], layer=layer, stage=self.s, tp_rank=self.t,
                   fault_time=time.time())
        self.event.close()
        os.kill(os.getpid(), signal.SIGKILL)

    # ------------------------------------------------------------------ main
    def run(self):
        a = self.args
        torch.set_num_threads(1)
        self.cfg = MoEConfig.tiny() if a.model == "tiny" else MoEConfig.bench()
        self.init_replica_groups()
        self.build_engine()
        eng = self.engine
        eng.optim.lr = a.lr
        eng.scheduler.base_lrs = [a.lr]
        eng.scheduler._last_lr = [a.lr]
        tok_loc = a.batch * a.seq_len // a.tp
        self.act_shape = (2, tok_loc, self.cfg.hidden)
        backend = a.backend or ("nccl" if self.device.type == "cuda" else "gloo")
        pg = ReconfigurableGroup(backend, a.communication_timeout, self.device if backend == "nccl" else None,
                                 prefix=f"x{self.rank}", event=self.event)
        transport = PackedTransport(pg, self.device if backend == "nccl" else torch.device("cpu"),
                                    timedelta(seconds=a.communication_timeout), self.event)
        store_port = int(os.environ.get("SHIFT_STORE_PORT", "0")) or _free_port()
        mode = WorldSizeMode.FIXED_WITH_SPARES if a.world_size_mode == "fixed_with_spares" else WorldSizeMode.DYNAMIC
        self.manager = Manager(pg, self.load_state, self.export_state, a.min_replicas, f"shift{a.replica}",
                               a.lighthouse, rank=self.rank, world_size=self.local_world,
                               store_addr=f"{a.host_ip}:{store_port}", hostname=a.host_ip,
                               checkpoint_transport=transport, timeout=timedelta(seconds=a.communication_timeout),
                               world_size_mode=mode, event=self.event)
        self.event("ready", hashes=self.current_hashes() if a.audit_state else {}, model=a.model,
                   params=eng.store.numel, device=str(self.device), stage=self.s, tp_rank=self.t,
                   placement=os.environ.get("SHIFT_CUDA_DEVICE", "cpu"))
        deadline = time.monotonic() + a.max_seconds
        while not self.marker("START").exists():
            if self.marker("STOP").exists() or time.monotonic() > deadline:
                raise RuntimeError("Stopped or timed out before START")
            time.sleep(0.02)
        self.loop_mp(deadline)

    def loop_mp(self, deadline):
        a, eng, mgr = self.args, self.engine, self.manager
        recovery_requested = False
        tokens_per_replica = a.microbatches * a.batch * a.seq_len
        while not self.requested_stop() and time.monotonic() < deadline and self.progress["updates"] < a.steps:
            it0 = time.monotonic()
            self.boundary_rng = dict(step=self.progress["updates"], rng=self.rng_snapshot())
            if a.generation > 0 and not recovery_requested:
                self.event("recovery_request", step=self.progress["updates"])
                recovery_requested = True
            mgr.start_quorum()
            step = self.progress["updates"]
            participants = mgr.num_participants()
            self.event("begin", step=step, participants=participants)
            loss = self.one_step(step)
            g = eng.store.grad
            if self.comm is not None and self.rep_end > 0:
                # TP-replicated parameters: the pair's partial gradients sum to the full one
                dist.all_reduce(g[: self.rep_end], group=self.tp_group)
            mgr.allreduce(g).wait()          # cross-replica average over the participants
            nonfinite = eng.optimizer_step([g], 1.0)
            if int(nonfinite.item()):
                mgr.report_error(RuntimeError("nonfinite gradients"))
            commit = mgr.should_commit()
            if commit:
                eng.commit()
                self.progress["updates"] += 1
                hashes = (self.current_hashes() if (a.hash_every and self.progress["updates"] % a.hash_every == 0)
                          else {})
                self.event("commit", step=self.progress["updates"], participants=mgr.num_participants(),
                           contributed=mgr.is_participating(), hashes=hashes, loss=loss,
                           tokens=tokens_per_replica * mgr.num_participants(), seconds=time.monotonic() - it0)
            else:
                self.event("skipped", step=step, error=str(mgr.errored()))
            if commit and self._replica_leaves(step):
                # GPU form of the fault: the rank leaves between steps, with
                # none of its kernels or collectives in flight.  Every rank of
                # the replica knows the plan, so the others stop at the same
                # boundary on the host instead of launching a step that would
                # wait for the dead rank inside a collective.
                if self.device.type == "cuda":
                    torch.cuda.synchronize(self.device)
                if self._kill_now(step, "sigkill_step"):
                    self._die(-1)
                self.event("replica_peer_leaving", step=self.progress["updates"], leaving_rank=a.inject_rank)
                self.event.close()
                os._exit(0)
        self.event("stopped", step=self.progress["updates"])
        mgr.shutdown()
        self.event.close()
        dist.destroy_process_group()


def main(argv=None):
    MPWorker(parse_args(argv)).run()


if __name__ == "__main__":
    main()
