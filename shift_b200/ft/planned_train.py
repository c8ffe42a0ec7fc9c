"""Role-aware trainer for planned handoff (roles A, B, C; variants p1f, p2).

    python -m shift_b200.ft.planned_train --planned-role A|B|C --planned-variant p1f|p2 \
        --coord HOST:PORT [trainer flags]

Epoch e uses the lighthouse at ``L + 10*e`` (``L + 10*e + 1`` for the A+B
fallback epoch of a rejected P2 relay) and Manager stores on their own ports,
as the reference moves to 31410 / 31411 (shift_full/planned_handoff.py:192,
shift_full/overlap_handoff.py:184-199).  A keeps logical replica id 0; B and
its replacement C both carry logical id 1, so C consumes exactly the data
B would have consumed (fixed batch).  Commit events carry the epoch and the
physical members.  Mirrors shift_full/planned_train.py.
"""
from __future__ import annotations

import os
import time
from datetime import timedelta

import torch

from ..engine import rng_state, set_rng_state
from .handoff import Coordinator, OverlapHandoff, PlannedHandoff
from .manager import Manager, WorldSizeMode
from .process_group import ReconfigurableGroup
from .train import Worker, _free_port, parse_args as base_parse
from .transport import PackedTransport


def parse_args(argv=None):
    import argparse
    extra = argparse.ArgumentParser(add_help=False)
    extra.add_argument("--planned-role", choices=["A", "B", "C"], required=True)
    extra.add_argument("--planned-variant", choices=["p0", "p1", "p1d", "p1f", "p2", "steady"], default="p1f")
    extra.add_argument("--planned-source", choices=["A", "B"], default="B")
    extra.add_argument("--planned-inject", default="healthy",
                       choices=["healthy", "prepare-fail", "ready-timeout", "stale-state", "relay-reject",
                                "slow-compute"])
    extra.add_argument("--planned-slow-ms", type=float, default=250)
    extra.add_argument("--planned-round", type=int, default=0)
    extra.add_argument("--planned-cycles", type=int, default=1,
                       help="rotation: rounds of the experiment; a process serves rounds [planned-round, cycles)")
    extra.add_argument("--coord", required=True)
    extra.add_argument("--mover", choices=["auto", "ipc", "packed"], default="auto")
    known, rest = extra.parse_known_args(argv)
    # each epoch's lighthouse address comes from the coordination store
    # (lighthouse/<slot>), so the base trainer's --lighthouse is a placeholder
    args = base_parse(rest + ["--lighthouse", "127.0.0.1:0"])
    for k, v in vars(known).items():
        setattr(args, k, v)
    return args


class PlannedWorker(Worker):
    # model-parallel subclasses reduce over the Manager's process group (NCCL)
    # instead of the fused peer-memory reducer of 1-GPU replicas
    group_reduce = False

    def __init__(self, args):
        super().__init__(args)
        self.role = args.planned_role
        self.logical_rid = 0 if self.role == "A" else 1
        self.round = args.planned_round
        self.forward_calls = 0

    def manifest(self):
        return {"numel": self.engine.store.numel, "specs": [(s.name, list(s.shape)) for s in self.engine.store.specs],
                "optimizer_groups": [{"betas": [self.engine.optim.beta1, self.engine.optim.beta2],
                                      "eps": self.engine.optim.eps, "weight_decay": self.engine.optim.weight_decay}]}

    def rng_tail(self):
        return dict(rng_state(self.device), progress=dict(self.progress), step=self.progress["updates"],
                    source_rank=self.rank)

    def apply_tail(self, tail):
        set_rng_state(tail, self.device)
        return tail

    # ------------------------------------------------------------------ managers per epoch
    def ensure_reducer(self):
        if getattr(self, "reducer", None) is None:
            from .fused import QuorumFusedReducer
            a = self.args
            self.reducer = QuorumFusedReducer(self.engine, self.device, self.role, a.generation, self.rank,
                                              a.communication_timeout, host=a.host_ip, event=self.event)
            layers = self.cfg.layers
            from ..parallel.replicas import _order
            self.engine.model.layer_done_hook = lambda layer: self.reducer.fused.on_layer_done(_order(layer, layers))
        return self.reducer

    # ------------------------------------------------------------------ preparation hooks (background)
    def premap_k1(self, handoff):
        """Exchange the fused-path buffers of the future AC pair now, so the
        first AC step only finds cached mappings."""
        if self.device.type != "cuda" or self.role not in ("A", "C"):
            return
        red = self.ensure_reducer()
        raw, pre = handoff.coord.raw, handoff.coord.prefix
        red.heap.publish(raw, make_default=False)
        raw.set(f"{pre}/k1owner/{self.role}/{self.rank}", red.owner)
        other = "C" if self.role == "A" else "A"
        key = f"{pre}/k1owner/{other}/{self.rank}"
        end = time.monotonic() + 600
        while not raw.check([key]):
            if time.monotonic() > end or handoff.coord.has("cancel"):
                return
            time.sleep(0.005)
        owner = raw.get(key).decode()
        for name in ("grad0", "grad1", "flags"):
            red.heap.open(owner, name, store=raw)
        self.event("planned_k1_premapped", peer=owner)

    def warmup_spare(self, handoff):
        """C: one forward/backward on a throw-away batch while A and B train,
        so the first real step pays no lazy initialisation (GPU standby).
        Touches only activations and the gradient buffer, never the state."""
        if self.role != "C":
            return
        from ..engine import synthetic_batch
        a = self.args
        data = synthetic_batch(self.cfg, 0, a.batch, a.seq_len, "pattern").to(self.device)
        self.engine.forward_backward([(data[:, :-1].contiguous(), data[:, 1:].contiguous())], a.batch, a.seq_len)
        self.engine.store.zero_grad()
        torch.cuda.synchronize(self.device)
        self.event("planned_spare_warm", seconds=0.0)

    def precreate_manager(self, handoff):
        if self.role in ("A", "C") and self.args.planned_variant in ("p1f", "p2"):
            self.next_manager = self.make_manager(handoff.new_epoch, "AC", activate=False)
            pg = getattr(self.next_manager, "_pg", None)
            # A (whose hooks do not wait for the spare) connects only once the
            # spare at its rank position is up, and not at all after a cancel
            ready = pg is not None and (self.role == "C" or handoff.coord.clone().wait(
                [f"local/C/{self.rank}"], 600, cancel_key="cancel"))
            if ready:
                # the A+C group of the next epoch (A is replica rank 0, the spare
                # takes replica 1's place), connected before the cut
                t0 = time.monotonic()
                try:
                    pg.prepare(self.coord.raw, f"e{handoff.new_epoch}/r{self.rank}", 0 if self.role == "A" else 1,
                               2)
                    self.event("planned_candidate_group_ready", epoch=handoff.new_epoch,
                               seconds=time.monotonic() - t0)
                except Exception as e:      # the epoch's quorum will build the group instead
                    self.event("planned_candidate_group_failed", epoch=handoff.new_epoch, error=repr(e))
            self.event("planned_candidate_manager_ready", epoch=handoff.new_epoch)

    def take_manager(self, epoch: int, members: str):
        m = getattr(self, "next_manager", None)
        if m is not None and members == "AC" and m._shift_epoch == epoch:
            self.next_manager = None
            m.load_state_dict({"step": self.progress["updates"]})
            self.manager = m
            return m
        return self.make_manager(epoch, members)

    def lighthouse_address(self, slot: int, timeout: float = 120.0) -> str:
        """Address of an epoch's lighthouse: the controller starts it on a port
        the OS chooses and publishes it under ``lighthouse/<slot>`` of the
        coordination store (slot = 10 * epoch, + 1 for a P2 round's fallback
        A+B epoch)."""
        key = f"lighthouse/{slot}"
        raw = self.coord.raw
        end = time.monotonic() + timeout
        while not raw.check([key]):
            if time.monotonic() > end:
                raise TimeoutError(f"no lighthouse published for slot {slot}")
            time.sleep(0.005)
        return raw.get(key).decode()

    def make_manager(self, epoch: int, members: str = "AB", activate: bool = True):
        a = self.args
        lighthouse = self.lighthouse_address(10 * epoch + (1 if members == "AB" and epoch > self.round else 0))
        if self.device.type == "cuda" and not self.group_reduce:
            # fused peer-memory reduction + IPC healing: a new epoch only re-maps handles
            from .fused import PeerStateTransport
            self.ensure_reducer()
            pg = None
            transport = PeerStateTransport(self.engine, self.device, self.reducer.owner, self.event,
                                           lambda: self.manager)
        else:
            cuda = self.device.type == "cuda"
            backend = a.backend or ("nccl" if cuda else "gloo")
            pg = ReconfigurableGroup(backend, a.communication_timeout, self.device if backend == "nccl" else None,
                                     prefix=f"x{self.rank}e{epoch}", event=self.event)
            transport = PackedTransport(pg, self.device if backend == "nccl" else torch.device("cpu"),
                                        timedelta(seconds=a.communication_timeout), self.event)
        rid = self.logical_rid
        store, store_addr = self.manager_store(epoch, members)
        m = Manager(pg, self.load_state_for_manager, self.export_state_for_transport, 2, f"shift{rid}",
                    lighthouse, rank=self.rank, world_size=self.local_world,
                    store_addr=store_addr, store=store, hostname=a.host_ip, checkpoint_transport=transport,
                    timeout=timedelta(seconds=a.communication_timeout),
                    world_size_mode=WorldSizeMode.FIXED_WITH_SPARES, event=self.event)
        m._shift_epoch = epoch
        m.load_state_dict({"step": self.progress["updates"]})   # a new epoch continues the committed step count
        if pg is None:
            m.on_quorum = lambda q, up, changed: (
                self.reducer.reconfigure(q, up, q.max_step) if changed or self.reducer.quorum_id != q.quorum_id
                else None)
            if activate:
                self.manager = m
        return m

    def manager_store(self, epoch: int, members: str):
        """(store, address) of the replica-local store of one epoch's Manager.
        Rank 0 lets the OS pick the port (a port computed ahead can be taken
        by then: every rank's process groups open sockets of their own); with
        several local ranks the port travels through the replica's own
        process-group store."""
        import torch.distributed as dist
        a = self.args
        t = timedelta(seconds=a.communication_timeout)
        key = f"planned_manager_store/{epoch}/{members}"
        shared = self.local_world > 1
        if shared and not dist.is_initialized():
            # no replica-local group to publish through: ports derived from the session's base
            base = int(os.environ.get("SHIFT_STORE_PORT", "0"))
            port = (base + 100 * (epoch + 1) + 7 * (members == "AB")) if base else _free_port()
            return None, f"{a.host_ip}:{port}"
        if self.rank == 0:
            store = dist.TCPStore(a.host_ip, 0, None, True, timeout=t, wait_for_workers=False)
            port = store.port
            if shared:
                dist.distributed_c10d._get_default_store().set(key, str(port))
        else:
            port = int(dist.distributed_c10d._get_default_store().get(key))
            store = dist.TCPStore(a.host_ip, port, None, False, timeout=t)
        return store, f"{a.host_ip}:{port}"

    def load_state(self, payload):
        if payload.get("_inplace"):
            # the state mover already wrote the flat buffers; apply the rest
            self.engine.scheduler.load_state_dict(payload["scheduler"])
            self.engine.store.step = int(payload["step"])
            self.progress.update(payload["progress"])
            set_rng_state(payload, self.device)
            hashes = self.current_hashes() if self.args.audit_state else {}
            ok = hashes == payload.get("hashes", {})
            self.event("restored", step=payload["step"], source_replica=payload["source_replica"],
                       source_rank=payload["source_rank"], hashes_match=ok, expected_hashes=payload.get("hashes"),
                       actual_hashes=hashes, mode="ipc")
            assert ok, "Restored state differs from source snapshot"
            return
        return super().load_state(payload)

    def batches(self, step):
        a = self.args
        out, ids = [], []
        from ..engine import synthetic_batch
        for micro in range(a.microbatches):
            sample = step * (a.microbatches * 4) + micro * 4 + self.logical_rid
            ids.append(sample)
            data = synthetic_batch(self.cfg, sample, a.batch, a.seq_len, a.data,
                                   seed_base=100_000 + a.data_seed * 1_000_000).to(self.device)
            out.append((data[:, :-1].contiguous(), data[:, 1:].contiguous()))
        return out, ids

    # ------------------------------------------------------------------ run
    def setup_engine(self):
        """The replica's model state (IPC-exportable on GPUs, so a spare can
        pull it straight from the donor's HBM)."""
        from ..engine import Engine
        a = self.args
        cuda = self.device.type == "cuda"
        self.engine = Engine(self.cfg, self.device, seed=a.seed, bucket_numel=a.bucket_size, ipc_state=cuda)
        if cuda:
            self.ensure_reducer()

    def compute(self, step, batches):
        """Forward + backward of this replica's share of step ``step``; the
        gradient is left in the engine's flat buffer."""
        return self.engine.forward_backward(batches, self.args.batch, self.args.seq_len)

    def run(self):
        from ..models.qwen_moe import MoEConfig
        a = self.args
        torch.set_num_threads(1)
        self.cfg = MoEConfig.tiny() if a.model == "tiny" else MoEConfig.bench()
        self.setup_engine()
        self.engine.optim.lr = a.lr
        self.engine.scheduler.base_lrs = [a.lr]
        self.engine.scheduler._last_lr = [a.lr]
        self.handoff = self.new_handoff(self.round)
        self.transport_on_cpu = False
        base_epoch = a.planned_round
        if self.role == "C":
            self.event("ready", role="C", planned_variant=a.planned_variant)
            ok = self.handoff.ready_receiver()
            if not ok:
                self.event("stopped", step=self.progress["updates"], role="C", cancelled=True)
                self.event.close()
                return
            self.manager = self.take_manager(base_epoch + 1, "AC")
            self.manager.load_state_dict({"step": self.progress["updates"]})
            self.event("planned_epoch_activated", step=self.progress["updates"], epoch=base_epoch + 1)
            self._advance_pending = True
        else:
            self.manager = self.make_manager(base_epoch, "AB")
            self.event("ready", role=self.role, planned_variant=a.planned_variant,
                       hashes=self.current_hashes() if a.audit_state else {})
            deadline = time.monotonic() + a.max_seconds
            while not self.marker("START").exists():
                if self.marker("STOP").exists() or time.monotonic() > deadline:
                    raise RuntimeError("Stopped or timed out before START")
                time.sleep(0.02)
        self.loop_planned(time.monotonic() + a.max_seconds)

    def new_handoff(self, round_: int):
        """The handoff protocol object of one rotation round (keys under
        ``round/<r>/`` of the coordination store, epochs r -> r+1)."""
        a = self.args
        cuda = self.device.type == "cuda"
        self.coord = Coordinator(a.coord, f"round/{round_}" if round_ else "")
        mover = a.mover if a.mover != "auto" else ("ipc" if cuda else "packed")
        cls = OverlapHandoff if a.planned_variant == "p2" else PlannedHandoff
        if self.group_reduce:           # model-parallel replicas: NCCL groups, per-stage warm-up
            hooks = [self.warmup_spare, self.precreate_manager]
        elif cuda:
            hooks = [self.premap_k1, self.warmup_spare, self.precreate_manager]
        else:
            hooks = [self.precreate_manager]
        emit = lambda kind, **kw: self.event(kind, round=round_, **kw)   # noqa: E731
        h = cls(self.role, a.planned_variant, self.rank, self.local_world, self.coord, emit,
                self.export_state, self.load_state, self.progress, self.manifest, self.device, mover,
                round_=round_, source=a.planned_source, inject=a.planned_inject if round_ == a.planned_round else
                "healthy", engine=self.engine, prepare_hooks=hooks)
        h.rng_tail = self.rng_tail
        return h

    def advance_round(self):
        """Continuous rotation (the reference's ``advance_round``): once epoch
        r+1 is active, the next round starts -- A stays A, the replica-1
        process that just took over becomes the donor B of round r+1, and a
        freshly launched spare will be its C."""
        if self.round + 1 >= self.args.planned_cycles:
            return
        self.round += 1
        if self.role == "C":
            self.role = "B"
        # the finished round still tracks its post-cut commits (the retired
        # donor of that round waits for them before it exits)
        self.prev_handoff = self.handoff
        self.handoff = self.new_handoff(self.round)
        self.event("planned_round_advanced", round=self.round, role=self.role, step=self.progress["updates"])

    def requested_stop(self):
        if super().requested_stop():
            return True
        m = self.marker("TRAIN_UNTIL")
        return m.exists() and self.progress["updates"] >= int(m.read_text().strip() or 0)

    def loop_planned(self, deadline):
        a, eng = self.args, self.engine
        attempts = 0
        while not self.requested_stop() and time.monotonic() < deadline and self.progress["updates"] < a.steps:
            it0 = time.monotonic()
            self.boundary_rng = dict(step=self.progress["updates"], rng=self.rng_snapshot())
            if self.role != "C":
                mgr, retired = self.handoff.boundary(self.manager)
                if retired:
                    self.event("stopped", step=self.progress["updates"], role=self.role, retired=True)
                    self.event.close()
                    return
                if mgr is None:
                    mgr = self.take_manager(self.handoff.gate.epoch, "AC")
                    mgr.load_state_dict({"step": self.progress["updates"]})
                    self.event("planned_epoch_activated", step=self.progress["updates"],
                               epoch=self.handoff.gate.epoch)
                    self.manager = mgr
                    self._advance_pending = True
                self.manager = mgr
            mgr = self.manager
            mgr.start_quorum()
            step = self.progress["updates"]
            self.event("begin", step=step, participants=mgr.num_participants())
            batches, sample_ids = self.batches(step)
            relay = a.planned_variant == "p2" and self.handoff.is_relay_step()
            fused = getattr(self, "reducer", None) is not None
            if fused:
                eng.nonfinite.zero_()
                self.reducer.before_step()
                self.reducer.fused.begin_step(step, defer=relay)
            t_c = time.monotonic()
            if relay and self.role == "C":
                eng.store.zero_grad()
                loss = torch.zeros(())
            else:
                loss = self.compute(step, batches)
                self.forward_calls += 1
                if a.planned_inject == "slow-compute":
                    time.sleep(a.planned_slow_ms / 1000.0)
            if relay:
                old_mgr = mgr
                mgr, retired = self.handoff.at_gradient(mgr, eng.store.grad, self.take_manager, sample_ids,
                                                        self.apply_tail)
                if retired:
                    self.event("stopped", step=self.progress["updates"], role=self.role, retired=True)
                    self.event.close()
                    return
                if mgr is not old_mgr and self.handoff.gate.epoch > self.handoff.base_epoch and \
                        not getattr(self.handoff, "fallback", False):
                    self._advance_pending = True       # A activated the new epoch inside the relay step
                self.manager = mgr
                self.event("planned_ac_outer_begin", step=step)
            if fused:
                nonfinite = self.reducer.fused.finish_step()
            else:
                mgr.allreduce(eng.store.grad).wait()
                nonfinite = eng.optimizer_step([eng.store.grad], 1.0)
            if int(nonfinite.item()):
                mgr.report_error(RuntimeError("nonfinite gradients"))
            commit = mgr.should_commit()
            attempts += 1
            if commit:
                eng.commit()
                self.progress["updates"] += 1
                hashes = self.current_hashes() if (a.hash_every and self.progress["updates"] % a.hash_every == 0) else {}
                self.event("commit", step=self.progress["updates"], participants=mgr.num_participants(),
                           contributed=mgr.is_participating(), hashes=hashes, sample_ids=sample_ids,
                           loss=float(loss), seconds=time.monotonic() - it0, compute_seconds=time.monotonic() - t_c,
                           forward_calls=self.forward_calls, relay_step=relay,
                           global_batch=a.batch * a.microbatches * mgr.num_participants(),
                           **self.handoff.commit_fields(mgr))
                self.handoff.committed()
                if getattr(self, "prev_handoff", None) is not None:
                    self.prev_handoff.committed()
                if getattr(self, "_advance_pending", False):
                    # the next rotation round starts after the first commit of the new epoch
                    self._advance_pending = False
                    self.advance_round()
            else:
                self.event("skipped", step=step, error=str(mgr.errored()))
        self.event("stopped", step=self.progress["updates"], attempts=attempts, role=self.role)
        self.handoff.cleanup_cancel.set()
        self.manager.shutdown()
        self.event.close()


def main(argv=None):
    args = parse_args(argv)
    PlannedWorker(args).run()


if __name__ == "__main__":
    main()
