"""Fault-tolerant per-rank trainer (one process per rank of one DP replica).

    python -m shift_b200.ft.train --session S --replica R --generation G \
        --lighthouse 127.0.0.1:PORT --root RESULTS [--model tiny|bench] [--device cpu|cuda] ...

Each step: quorum (heal from a live peer if this replica is behind) ->
synthetic microbatches -> forward/backward -> cross-replica gradient average
(participants only; a healing replica contributes zeros) -> non-finite check
-> commit vote -> AdamW into the next state generation -> commit flips it.
Events go to ``<root>/<session>/events_g<generation>_r<rank>.jsonl`` with the
reference worker's kinds (ready, phase, begin, commit, skipped, snapshot,
state_loaded, restored, recovery_request, transport_send/recv,
checkpoint_saved/loaded/resumed, standby_ready/activated, stopped) --
shift_full/train.py:124-627.  Marker files in the session directory: START
(begin training), STOP (optionally holding a step bound), ACTIVATE (leave
standby).

Gradient path: ``--reduce fused`` (CUDA) runs the cross-replica reduction
inside the fused AdamW kernel over peer memory; ``--reduce group`` averages
the flat gradient with the Manager's process group first (gloo on CPU, NCCL on
GPU) -- the baseline.
"""
from __future__ import annotations

import argparse
import os
import random
import time
from datetime import timedelta
from pathlib import Path

_MODULE_STARTED = time.monotonic()

import torch  # noqa: E402

from ..engine import Engine, rng_state, set_rng_state, synthetic_batch  # noqa: E402
from ..models.qwen_moe import MoEConfig  # noqa: E402
from ..utils.digest import cpu_tree, digest, tensor_count  # noqa: E402
from ..utils.events import EventLog  # noqa: E402
from .manager import Manager, WorldSizeMode  # noqa: E402
from .process_group import ReconfigurableGroup  # noqa: E402
from .transport import PackedTransport  # noqa: E402


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--session", required=True)
    p.add_argument("--replica", type=int, required=True)
    p.add_argument("--generation", type=int, default=0)
    p.add_argument("--host-ip", default="127.0.0.1")
    p.add_argument("--lighthouse", required=True)
    p.add_argument("--root", default="results")
    p.add_argument("--max-seconds", type=int, default=900)
    p.add_argument("--model", choices=["tiny", "bench"], default="tiny")
    p.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    p.add_argument("--backend", choices=["gloo", "nccl"], default=None)
    p.add_argument("--reduce", choices=["group", "fused"], default="group")
    p.add_argument("--steps", "--target-steps", dest="steps", type=int, default=1_000_000)
    p.add_argument("--seq-len", type=int, default=128)
    p.add_argument("--batch", type=int, default=4, help="sequences per microbatch")
    p.add_argument("--microbatches", type=int, default=1)
    p.add_argument("--hash-every", type=int, default=0)
    p.add_argument("--audit-state", action="store_true")
    p.add_argument("--audit-hash", choices=["sha256", "sha256tree", "fingerprint"], default="sha256",
                   help="sha256: the reference's host digest of the state dict; sha256tree: SHA-256 over the "
                        "SHA-256 digests of 64 KiB leaves of the flat state, computed on the GPU; fingerprint: "
                        "64-bit FNV-1a of the flat state on the GPU")
    p.add_argument("--fixed-batch", action="store_true")
    p.add_argument("--data", choices=["pattern", "random"], default="random")
    p.add_argument("--data-seed", type=int, default=0, help="uniform random ids from seed data_seed*1e6+sample")
    p.add_argument("--lr", type=float, default=1e-4)
    p.add_argument("--min-replicas", type=int, default=1)
    p.add_argument("--world-size-mode", choices=["dynamic", "fixed_with_spares"], default="dynamic")
    p.add_argument("--communication-timeout", type=float, default=30)
    p.add_argument("--checkpoint-step", type=int, default=0)
    p.add_argument("--checkpoint-cold", action="store_true")
    p.add_argument("--resume-checkpoint", action="store_true")
    p.add_argument("--standby", choices=("cpu", "gpu"))
    p.add_argument("--lazy-init", action="store_true",
                   help="skip the seeded initialisation: the state must come from a live peer at the first quorum "
                        "(a relaunched replica); the worker refuses to train otherwise")
    p.add_argument("--activate-marker", default="ACTIVATE",
                   help="marker file (in the session directory) that releases a standby process")
    p.add_argument("--bucket-size", type=int, default=64 * 1024 * 1024)
    p.add_argument("--inject", default="", help="test fault: nonfinite@STEP | exit@STEP | slow@MS")
    p.add_argument("--mode", choices=["shift", "flat"], default="shift",
                   help="flat: one process trains the whole global batch of --flat-replicas data ranks, "
                        "no Manager (the non-fault-tolerant numerical baseline)")
    p.add_argument("--flat-replicas", type=int, default=2)
    p.add_argument("--reference-dump", default="",
                   help="comma-separated committed steps after which the averaged gradient, model, optimizer and "
                        "scheduler are saved to reference_step<k>_r<rank>.pt (group reduction or flat mode)")
    p.add_argument("--profile-timings", action="store_true",
                   help="split the cross-replica phase of each step: device time between CUDA events around it "
                        "(cross_gpu_seconds) and host time to copy, dispatch and wait")
    p.add_argument("--trace-routing", action="store_true",
                   help="also log a 'routing' event per step, sample and MoE layer with the digest of the router's "
                        "top-k expert indices (read by shift_b200.analysis.trajectory)")
    p.add_argument("--reference-anchor", default="",
                   help="start from another run's reference dump: the directory holding reference_step<k>_r<rank>.pt")
    p.add_argument("--reference-anchor-step", type=int, default=0,
                   help="k of the anchor dump; training continues at step k with that model, optimizer and scheduler")
    p.add_argument("--seed", type=int, default=2026)
    return p.parse_args(argv)


class Worker:
    def __init__(self, args):
        self.args = args
        self.rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.local_world = int(os.environ.get("LOCAL_WORLD_SIZE", os.environ.get("WORLD_SIZE", "1")))
        self.out = Path(os.environ.get("SHIFT_RESULT_DIR", str(Path(args.root) / args.session)))
        self.out.mkdir(parents=True, exist_ok=True)
        self.event = EventLog(self.out / f"events_g{args.generation}_r{self.rank}.jsonl", rid=args.replica,
                              rank=self.rank, generation=args.generation,
                              physical_node=os.environ.get("SHIFT_PHYSICAL_NODE", args.host_ip), host_ip=args.host_ip)
        self.event.keep = False
        if args.device == "cuda":
            dev_index = int(os.environ.get("SHIFT_CUDA_DEVICE", self.rank))
            torch.cuda.set_device(dev_index)
            self.device = torch.device("cuda", dev_index)
        else:
            self.device = torch.device("cpu")
        self.progress = {"updates": 0}
        self.manager = None
        self.boundary_rng = None

    # ------------------------------------------------------------------ helpers
    def phase(self, name, started):
        self.event("phase", name=name, seconds=time.monotonic() - started)
        return time.monotonic()

    def marker(self, name) -> Path:
        return self.out / name

    def standby_gate(self, mode):
        import resource
        self.event("standby_ready", mode=mode, cpu_maxrss_kib=resource.getrusage(resource.RUSAGE_SELF).ru_maxrss,
                   cuda_allocated_bytes=torch.cuda.memory_allocated() if self.device.type == "cuda" else 0)
        until = time.monotonic() + self.args.max_seconds
        while not self.marker(self.args.activate_marker).exists():
            if self.marker("STOP").exists() or time.monotonic() > until:
                raise RuntimeError("standby stopped or timed out before activation")
            time.sleep(0.02)
        self.event("standby_activated", mode=mode)

    def rng_snapshot(self):
        return rng_state(self.device)

    def current_hashes(self, rng=None):
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        rng = rng if rng is not None else self.rng_snapshot()
        mode = getattr(self.args, "audit_hash", "sha256")
        if mode == "sha256tree":
            # SHA-256 of every 64 KiB leaf of the flat state buffers, computed
            # where the state lives (a GPU kernel on CUDA), then SHA-256 over
            # the leaf digests: the full-state audit without a host copy
            from ..utils.digest import sha256tree
            st = self.engine.store
            c = st.cur
            opt = "/".join(sha256tree(t[c]) for t in (st.master, st.exp_avg, st.exp_avg_sq))
            return dict(model="st:" + sha256tree(st.param[c]), optimizer=f"st:{opt}/{st.step}",
                        scheduler=digest(self.engine.scheduler.state_dict()), progress=digest(self.progress),
                        cpu_rng=digest(rng["torch_rng"]), cuda_rng=digest(rng["cuda_rng"]),
                        python_rng=digest(rng["python_rng"]))
        if mode == "fingerprint" and self.device.type == "cuda":
            # exact-state fingerprints computed on the GPU (no host copy of the state)
            from ..ops._ext import ext
            st = self.engine.store
            c = st.cur
            opt = "/".join(ext().fingerprint(t[c]) for t in (st.master, st.exp_avg, st.exp_avg_sq))
            return dict(model="fp:" + ext().fingerprint(st.param[c]), optimizer=f"fp:{opt}/{st.step}",
                        scheduler=digest(self.engine.scheduler.state_dict()), progress=digest(self.progress),
                        cpu_rng=digest(rng["torch_rng"]), cuda_rng=digest(rng["cuda_rng"]),
                        python_rng=digest(rng["python_rng"]))
        sd = self.engine.state_dict()
        return dict(model=digest(sd["model"]), optimizer=digest(sd["optimizer"]), scheduler=digest(sd["scheduler"]),
                    progress=digest(self.progress), cpu_rng=digest(rng["torch_rng"]), cuda_rng=digest(rng["cuda_rng"]),
                    python_rng=digest(rng["python_rng"]))

    # ------------------------------------------------------------------ state
    def export_state(self):
        self.event("snapshot_begin", step=self.progress["updates"])
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        step = self.manager.current_step() if self.manager else self.progress["updates"]
        assert step == self.progress["updates"], (step, self.progress)
        rng = (self.boundary_rng["rng"] if self.boundary_rng and self.boundary_rng["step"] == step
               else self.rng_snapshot())
        sd = self.engine.state_dict()
        payload = dict(model=sd["model"], optimizer=sd["optimizer"], scheduler=sd["scheduler"],
                       progress=dict(self.progress), **rng, source_replica=self.args.replica, source_rank=self.rank,
                       step=step)
        payload["hashes"] = self.current_hashes(rng) if self.args.audit_state else {}
        self.event("snapshot", step=step, hashes=payload["hashes"],
                   optimizer_tensors=tensor_count(payload["optimizer"].get("state", {})))
        return payload

    def load_state(self, payload):
        t0 = time.monotonic()
        assert payload["source_rank"] == self.rank, (payload["source_rank"], self.rank)
        assert payload["step"] == payload["progress"]["updates"]
        if self.manager:
            assert payload["step"] == self.manager.current_step()
        if payload.get("_inplace"):
            # flat buffers were already copied from the donor's HBM; apply the rest
            self.engine.scheduler.load_state_dict(payload["scheduler"])
            self.engine.store.step = int(payload["step"])
        else:
            self.engine.load_state_dict(payload)
        self.progress.update(payload["progress"])
        set_rng_state(payload, self.device)
        self.healed = True
        if self.device.type == "cuda":
            torch.cuda.current_stream().synchronize()
        loaded = time.monotonic()
        self.event("state_loaded", step=payload["step"], load_seconds=loaded - t0,
                   source_replica=payload["source_replica"], source_rank=payload["source_rank"])
        hashes = self.current_hashes() if self.args.audit_state else {}
        matches = hashes == payload["hashes"]
        self.event("restored", step=payload["step"], load_seconds=loaded - t0, audit_seconds=time.monotonic() - loaded,
                   source_replica=payload["source_replica"], source_rank=payload["source_rank"], hashes_match=matches,
                   expected_hashes=payload["hashes"], actual_hashes=hashes)
        assert matches, "Restored state differs from source snapshot"

    # ------------------------------------------------------------------ data
    def batches(self, step):
        a = self.args
        ranks = range(a.flat_replicas) if a.mode == "flat" else [a.replica]
        out, ids = [], []
        for data_rank in ranks:
            for micro in range(a.microbatches):
                sample = step * (a.microbatches * 4) + micro * 4 + data_rank
                ids.append(sample)
                data = synthetic_batch(self.cfg, sample, a.batch, a.seq_len, a.data,
                                       seed_base=100_000 + a.data_seed * 1_000_000)
                data = data.to(self.device, non_blocking=True)
                out.append((data[:, :-1].contiguous(), data[:, 1:].contiguous()))
        return out, ids

    def forward_backward(self, batches, ids, step):
        """One step's forward/backward over its microbatches, with the
        evidence the trajectory summary compares across runs: a 'batch_plan'
        event (the sample ids of the step, before the update) and, with
        --trace-routing, one 'routing' event per sample and MoE layer holding
        the digest of the router's top-k expert indices."""
        a, eng = self.args, self.engine
        self.event("batch_plan", step=step, sample_ids=ids)
        if not a.trace_routing:
            return eng.forward_backward(batches, a.batch, a.seq_len)
        seen = []
        eng.model.routing_hook = lambda layer, idx: seen.append((layer, digest(idx)))
        try:
            loss = eng.forward_backward(batches, a.batch, a.seq_len)
        finally:
            eng.model.routing_hook = None
        per = len(seen) // max(1, len(ids))      # microbatch m runs sample ids[m] through every layer
        for m, sample in enumerate(ids):
            for layer, h in seen[m * per:(m + 1) * per]:
                self.event("routing", step=step, sample=sample, layer=layer, topk_hash=h)
        return loss

    def load_anchor(self):
        """Continue from the committed state of another run's reference dump
        (model, optimizer, scheduler after step k; the reference's
        --reference-anchor): two runs anchored at the same dump start from
        identical bits, so their next steps' routing and gradients can be
        compared without the drift of earlier steps."""
        a = self.args
        path = Path(a.reference_anchor) / f"reference_step{a.reference_anchor_step}_r{self.rank}.pt"
        dump = torch.load(path, map_location="cpu", weights_only=False)
        assert int(dump["step"]) == a.reference_anchor_step, (dump["step"], a.reference_anchor_step)
        self.engine.load_state_dict(_to_device({k: dump[k] for k in ("model", "optimizer", "scheduler")},
                                               self.device))
        self.progress["updates"] = int(dump["step"])
        if self.manager is not None:
            self.manager.load_state_dict({"step": int(dump["step"])})
        self.event("reference_anchor_loaded", step=int(dump["step"]), source=str(path))

    def reference_dump(self, grad):
        """Per-step numerical reference (shift_full/train.py:584-587 semantics):
        the averaged gradient and the committed state after the step."""
        steps = {int(x) for x in self.args.reference_dump.split(",") if x.strip()}
        if self.progress["updates"] not in steps:
            return
        sd = self.engine.state_dict()
        payload = cpu_tree(dict(step=self.progress["updates"], gradients=grad.detach().float(),
                                model=sd["model"], optimizer=sd["optimizer"], scheduler=sd["scheduler"],
                                offsets={k: [int(o), list(sh)] for k, (o, sh) in self.engine.store.offsets.items()}))
        torch.save(payload, self.out / f"reference_step{self.progress['updates']}_r{self.rank}.pt")
        self.event("reference_dump", step=self.progress["updates"])

    def run_flat(self):
        """The flat baseline: no quorum, no Manager; one replica trains every
        data rank's microbatches (the same global batch as the shift run)."""
        a = self.args
        if a.reference_anchor:
            self.load_anchor()
        self.event("ready", model=a.model, mode="flat", params=self.engine.store.numel,
                   hashes=self.current_hashes() if a.audit_state else {})
        eng = self.engine
        while self.progress["updates"] < a.steps and not self.requested_stop():
            it0 = time.monotonic()
            batches, ids = self.batches(self.progress["updates"])
            loss = self.forward_backward(batches, ids, self.progress["updates"])
            g = eng.store.grad
            eng.optimizer_step([g], 1.0)
            grad_copy = g.detach().clone() if a.reference_dump else None
            eng.commit()
            self.progress["updates"] += 1
            if a.reference_dump:
                self.reference_dump(grad_copy)
            self.event("commit", step=self.progress["updates"], participants=1, loss=float(loss), sample_ids=ids,
                       seconds=time.monotonic() - it0)
        self.event("stopped", step=self.progress["updates"])
        self.event.close()

    # ------------------------------------------------------------------ main
    def run(self):
        a = self.args
        if a.standby == "cpu":
            self.standby_gate("cpu")
        started = self.phase("python_imports", _MODULE_STARTED)
        torch.set_num_threads(1)
        self.cfg = MoEConfig.tiny() if a.model == "tiny" else MoEConfig.bench()
        self.engine = Engine(self.cfg, self.device, seed=a.seed, bucket_numel=a.bucket_size, init=not a.lazy_init)
        self.engine.optim.lr = a.lr
        self.engine.scheduler.base_lrs = [a.lr]
        self.engine.scheduler._last_lr = [a.lr]
        started = self.phase("model_load", started)
        if a.mode == "flat":
            return self.run_flat()
        if a.standby == "gpu":
            self.standby_gate("gpu")
        backend = a.backend or ("nccl" if self.device.type == "cuda" else "gloo")
        self.reducer = None
        if a.reduce == "fused":
            if self.device.type != "cuda":
                raise ValueError("--reduce fused needs a CUDA device")
            from .fused import PeerStateTransport, QuorumFusedReducer
            self.reducer = QuorumFusedReducer(self.engine, self.device, f"shift{a.replica}", a.generation, self.rank,
                                              a.communication_timeout, host=a.host_ip, event=self.event)
            layers = self.cfg.layers
            from ..parallel.replicas import _order
            self.engine.model.layer_done_hook = lambda layer: self.reducer.fused.on_layer_done(_order(layer, layers))
            pg = None
            transport = PeerStateTransport(self.engine, self.device, self.reducer.owner, self.event,
                                           lambda: self.manager)
            backend = "peer-ipc"
        else:
            pg = ReconfigurableGroup(backend, a.communication_timeout, self.device if backend == "nccl" else None,
                                     prefix=f"x{self.rank}", event=self.event)
            transport = PackedTransport(pg, self.device if backend == "nccl" else torch.device("cpu"),
                                        timedelta(seconds=a.communication_timeout), self.event)
        store_port = int(os.environ.get("SHIFT_STORE_PORT", "0")) or _free_port()
        mode = WorldSizeMode.FIXED_WITH_SPARES if a.world_size_mode == "fixed_with_spares" else WorldSizeMode.DYNAMIC
        self.manager = Manager(pg, self.load_state_for_manager, self.export_state_for_transport, a.min_replicas,
                               f"shift{a.replica}", a.lighthouse, rank=self.rank, world_size=self.local_world,
                               store_addr=f"{a.host_ip}:{store_port}", hostname=a.host_ip,
                               checkpoint_transport=transport, timeout=timedelta(seconds=a.communication_timeout),
                               world_size_mode=mode, event=self.event)
        if self.reducer is not None:
            self.manager.on_quorum = lambda q, up, changed: (
                self.reducer.reconfigure(q, up, q.max_step) if changed or self.reducer.quorum_id is None else None)
        self.transport_on_cpu = backend == "gloo" and self.device.type == "cuda"
        started = self.phase("manager_init", started)
        if a.resume_checkpoint:
            self.resume()
        if a.reference_anchor:
            self.load_anchor()
        self.event("ready", hashes=self.current_hashes() if a.audit_state else {}, model=a.model,
                   params=self.engine.store.numel, device=str(self.device), backend=backend, reduce=a.reduce,
                   full_parameters=self.cfg.param_count())
        deadline = time.monotonic() + a.max_seconds
        while not self.marker("START").exists():
            if self.marker("STOP").exists() or time.monotonic() > deadline:
                raise RuntimeError("Stopped or timed out before START")
            time.sleep(0.02)
        self.loop(deadline)

    def load_state_for_manager(self, payload):
        if self.device.type == "cuda" and getattr(self, "transport_on_cpu", False):
            payload = _to_device(payload, self.device)
        self.load_state(payload)

    def export_state_for_transport(self):
        p = self.export_state()
        if getattr(self, "transport_on_cpu", False):
            p = cpu_tree(p)
        return p

    def requested_stop(self):
        m = self.marker("STOP")
        if not m.exists():
            return False
        text = m.read_text().strip()
        return not text or self.progress["updates"] >= int(text)

    def loop(self, deadline):
        a, eng, mgr = self.args, self.engine, self.manager
        attempts = 0
        inject_kind, _, inject_arg = a.inject.partition("@")
        recovery_requested = False
        while not self.requested_stop() and time.monotonic() < deadline and self.progress["updates"] < a.steps:
            it0 = time.monotonic()
            if self.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
            self.boundary_rng = dict(step=self.progress["updates"], rng=self.rng_snapshot())
            if a.generation > 0 and not recovery_requested:
                self.event("recovery_request", step=self.progress["updates"])
                recovery_requested = True
            q0 = time.monotonic()
            mgr.start_quorum()
            if a.lazy_init and not getattr(self, "healed", False):
                raise RuntimeError("--lazy-init: the first quorum did not load a live peer's state into this replica")
            step = self.progress["updates"]
            participants = mgr.num_participants()
            self.event("begin", step=step, participants=participants, quorum_seconds=time.monotonic() - q0)
            if inject_kind == "exit" and step == int(inject_arg):
                self.event("injected_exit", step=step)
                os._exit(17)
            batches, sample_ids = self.batches(step)
            t_compute = time.monotonic()
            schedule_s = t_compute - it0
            if self.reducer is not None:
                eng.nonfinite.zero_()
                self.reducer.before_step()
                self.reducer.fused.begin_step(step)
            loss = self.forward_backward(batches, sample_ids, step)
            if inject_kind == "slow":
                time.sleep(float(inject_arg) / 1000.0)
            if inject_kind == "nonfinite" and step == int(inject_arg):
                eng.store.grad.view(-1)[0] = float("nan")
            # cross-replica average (participants only)
            prof = {}
            cuda_prof = a.profile_timings and self.device.type == "cuda"
            if cuda_prof:
                ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ev0.record()
            t_cross = time.monotonic()
            if a.reduce == "group":
                g = eng.store.grad
                if self.transport_on_cpu:
                    gc = g.float().cpu()
                    t_copied = time.monotonic()
                    work = mgr.allreduce(gc)
                    t_issued = time.monotonic()
                    work.wait()
                    g.copy_(gc)
                else:
                    t_copied = time.monotonic()
                    work = mgr.allreduce(g)
                    t_issued = time.monotonic()
                    work.wait()
                t_waited = time.monotonic()
                prof = dict(d2h_seconds=t_copied - t_cross, dispatch_seconds=t_issued - t_copied,
                            wait_seconds=t_waited - t_issued)
                nonfinite = eng.optimizer_step([g], 1.0)
            else:
                # reduction + AdamW already ran per bucket inside the fused kernel
                nonfinite = self.reducer.fused.finish_step()
            if cuda_prof:
                ev1.record()
            t_check = time.monotonic()
            finite = int(nonfinite.item()) == 0
            gradient_check_s = time.monotonic() - t_check
            if cuda_prof:
                prof["cross_gpu_seconds"] = ev0.elapsed_time(ev1) / 1000.0
            if a.profile_timings:
                prof["cross_host_seconds"] = t_check - t_cross
            if not finite:
                mgr.report_error(RuntimeError("nonfinite gradients"))
            if self.reducer is not None:
                from ..ops._ext import status_word
                sw = status_word(self.device)
                if int(sw[0].item()) != 0:
                    mgr.report_error(RuntimeError(f"fused path status {int(sw[0].item())}"))
                    sw.zero_()
            t_decide = time.monotonic()
            commit = mgr.should_commit()
            attempts += 1
            if commit:
                eng.commit()
                self.progress["updates"] += 1
                hashes = (self.current_hashes() if (a.hash_every and self.progress["updates"] % a.hash_every == 0)
                          else {})
                self.event("commit", step=self.progress["updates"], updates=self.progress["updates"],
                           participants=mgr.num_participants(), contributed=mgr.is_participating(), hashes=hashes,
                           model_hash=hashes.get("model"), optimizer_hash=hashes.get("optimizer"),
                           scheduler_hash=hashes.get("scheduler"), sample_ids=sample_ids, finite_gradients=finite,
                           loss=float(loss), seconds=time.monotonic() - it0, compute_seconds=t_decide - t_compute,
                           decision_seconds=time.monotonic() - t_decide, schedule_seconds=schedule_s,
                           gradient_check_seconds=gradient_check_s, **prof,
                           global_batch=a.batch * a.microbatches * mgr.num_participants())
            else:
                self.event("skipped", step=step, error=str(mgr.errored()), finite_gradients=finite)
            assert mgr.current_step() == self.progress["updates"]
            if a.checkpoint_step and self.progress["updates"] == a.checkpoint_step and commit:
                self.save_checkpoint()
            if commit and a.reference_dump and a.reduce == "group":
                self.reference_dump(eng.store.grad)
        self.event("stopped", step=self.progress["updates"], attempts=attempts)
        if self.reducer is not None:
            self.reducer.close()
        mgr.shutdown()
        self.event.close()

    # ------------------------------------------------------------------ disk checkpoint baseline
    def checkpoint_path(self) -> Path:
        """One file per replica and rank (the replicas of a session share its directory)."""
        return self.out / f"checkpoint_rid{self.args.replica}_r{self.rank}.pt"

    def save_checkpoint(self):
        t0 = time.monotonic()
        payload = cpu_tree(self.export_state())
        path = self.checkpoint_path()
        tmp = path.with_name(path.name + f".tmp{os.getpid()}")
        torch.save(payload, tmp)
        with tmp.open("rb") as h:
            os.fsync(h.fileno())
        os.replace(tmp, path)          # replicas share the session directory: write whole files only
        self.event("checkpoint_saved", step=self.progress["updates"], seconds=time.monotonic() - t0,
                   bytes=path.stat().st_size)
        t1 = time.monotonic()
        loaded = torch.load(path, weights_only=False)
        self.engine.load_state_dict(_to_device(loaded, self.device))
        self.event("checkpoint_loaded", step=self.progress["updates"], seconds=time.monotonic() - t1,
                   cache="warm_after_save",
                   hashes_match=not self.args.audit_state or self.current_hashes() == payload.get("hashes"))
        if self.args.checkpoint_cold:
            with path.open("rb") as h:
                os.posix_fadvise(h.fileno(), 0, 0, os.POSIX_FADV_DONTNEED)
            t2 = time.monotonic()
            loaded = torch.load(path, weights_only=False)
            self.engine.load_state_dict(_to_device(loaded, self.device))
            self.event("checkpoint_loaded_cold", step=self.progress["updates"], seconds=time.monotonic() - t2,
                       cache="fadvise_dontneed_advisory")

    def resume(self):
        path = self.checkpoint_path()
        t0 = time.monotonic()
        payload = torch.load(path, weights_only=False)
        self.engine.load_state_dict(_to_device(payload, self.device))
        self.progress.update(payload["progress"])
        set_rng_state(payload, self.device)
        self.manager.load_state_dict({"step": payload["step"]})
        self.event("checkpoint_resumed", step=payload["step"], seconds=time.monotonic() - t0)


def _to_device(tree, device):
    if isinstance(tree, torch.Tensor):
        return tree.to(device) if tree.is_floating_point() or tree.dtype in (torch.int32, torch.int64) else tree
    if isinstance(tree, dict):
        return {k: (_to_device(v, device) if k not in ("torch_rng", "cuda_rng") else v) for k, v in tree.items()}
    if isinstance(tree, list):
        return [_to_device(v, device) for v in tree]
    if isinstance(tree, tuple):
        return tuple(_to_device(v, device) for v in tree)
    return tree


def _free_port() -> int:
    import socket
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def main(argv=None):
    args = parse_args(argv)
    random.seed(args.seed + args.replica)
    Worker(args).run()


if __name__ == "__main__":
    main()
