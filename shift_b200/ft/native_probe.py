"""Model-free fault-tolerance probe: one large parameter, no model.

    python -m shift_b200.control.launch --nproc 1 --module shift_b200.ft.native_probe -- \
        --session S --replica R --lighthouse HOST:PORT [--numel 125000000] [--device cuda] [--steps N]

Each step: quorum -> deterministic gradient (seeded by step and replica, the
same on every run) -> cross-replica average through the Manager -> AdamW on
the flat fp32 master / moments -> commit vote.  It measures what the
fault-tolerance layer itself costs (quorum, reduction, optimizer, state size)
without the model's compute -- the reference's native probe
(shift_full/native_probe.py: one bf16 parameter of 125M elements,
manager.allreduce, Adam).  Events: ready (state bytes), commit (quorum /
reduce / optimizer seconds), stopped.  Runs under the same supervisors and
markers as the trainer, so a kill / heal of the probe exercises the same
recovery path with a 1-parameter state.

It also probes two building blocks of the planned handoff in isolation (the
reference's linear-layer probes sf/planned_probe.py and sf/planned_overlap.py):

* ``--world-size-mode fixed_with_spares --min-replicas K``: replicas beyond
  the first K at the quorum's step are spares -- they take part in every
  reduction with a zero contribution and apply the average, so a spare's
  state follows the participants' bit for bit without changing the result
  (the shadow a planned spare keeps before it takes over);
* ``--snapshot-overlap``: every step copies the committed generation of the
  state (parameters, fp32 master, both moments) into a snapshot buffer
  while the step's gradient, reduction and AdamW run -- on a side CUDA stream,
  or a host thread on CPU.  The flat ping-pong buffers make that generation
  read-only during the step (AdamW writes the other one); the probe checks it
  (tensor version counters) and that the snapshot equals the state it copied
  (the pre-copy window of the P2 handoff).
"""
from __future__ import annotations

import os
import threading
import time
from datetime import timedelta

import torch

from ..engine import Engine
from ..models.qwen_moe import MoEConfig
from ..parallel.flat import ParamSpec
from .manager import Manager, WorldSizeMode
from .process_group import ReconfigurableGroup
from .train import Worker, _free_port, parse_args as base_parse
from .transport import PackedTransport


def parse_args(argv=None):
    import argparse
    extra = argparse.ArgumentParser(add_help=False, allow_abbrev=False)
    extra.add_argument("--numel", type=int, default=125_000_000)
    extra.add_argument("--snapshot-overlap", action="store_true")
    known, rest = extra.parse_known_args(argv)
    args = base_parse(rest)
    args.numel = known.numel
    args.snapshot_overlap = known.snapshot_overlap
    return args


class _Snapshot:
    """Copy of one generation of the flat state, taken concurrently with a step."""

    def __init__(self, store, device):
        self.store, self.device = store, device
        self.bufs = None
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def _sources(self):
        st, c = self.store, self.store.cur
        return [st.param[c], st.master[c], st.exp_avg[c], st.exp_avg_sq[c]]

    def begin(self):
        src = self._sources()
        if self.bufs is None:
            self.bufs = [torch.empty_like(t) for t in src]
        self.versions = [t._version for t in src]
        self.t0 = time.monotonic()
        if self.stream is not None:
            self.stream.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.stream):
                for b, t in zip(self.bufs, src):
                    b.copy_(t, non_blocking=True)
                self.done = torch.cuda.Event()
                self.done.record(self.stream)
            self.thread = None
        else:
            def work():
                for b, t in zip(self.bufs, src):
                    b.copy_(t)
                self.copy_end = time.monotonic()
            self.thread = threading.Thread(target=work, daemon=True)
            self.thread.start()
        return src

    def finish(self, src) -> dict:
        """After the step (before commit flips the generation)."""
        if self.thread is not None:
            self.thread.join()
            copy_s = self.copy_end - self.t0
        else:
            self.done.synchronize()
            copy_s = time.monotonic() - self.t0
        unchanged = [t._version for t in src] == self.versions
        equal = all(torch.equal(b, t) for b, t in zip(self.bufs, src))
        return {"copy_seconds": copy_s, "window_seconds": time.monotonic() - self.t0,
                "source_unchanged": unchanged, "snapshot_equal": equal,
                "bytes": sum(t.numel() * t.element_size() for t in src)}


class ProbeWorker(Worker):
    def gradient(self, step):
        g = torch.Generator(device="cpu").manual_seed(1_000_003 * step + 7919 * self.args.replica)
        n = self.engine.store.numel
        # a cheap deterministic pattern: one random scale per step and replica over a fixed ramp
        scale = float(torch.rand((), generator=g)) * 1e-3
        ramp = torch.linspace(-1.0, 1.0, n, device=self.device, dtype=torch.float32)
        return (ramp * scale).to(self.engine.store.compute_dtype)

    def run(self):
        a = self.args
        cfg = MoEConfig.tiny()                       # only for the engine's bookkeeping; no model is run
        specs = [ParamSpec("probe.weight", (a.numel,))]
        self.engine = Engine(cfg, self.device, specs=specs, bucket_numel=a.bucket_size)
        st = self.engine.store
        backend = a.backend or ("nccl" if self.device.type == "cuda" else "gloo")
        pg = ReconfigurableGroup(backend, a.communication_timeout, self.device if backend == "nccl" else None,
                                 prefix=f"x{self.rank}", event=self.event)
        transport = PackedTransport(pg, self.device if backend == "nccl" else torch.device("cpu"),
                                    timedelta(seconds=a.communication_timeout), self.event)
        store_port = int(os.environ.get("SHIFT_STORE_PORT", "0")) or _free_port()
        self.manager = Manager(pg, self.load_state, self.export_state, a.min_replicas, f"shift{a.replica}",
                               a.lighthouse, rank=self.rank, world_size=self.local_world,
                               store_addr=f"{a.host_ip}:{store_port}", hostname=a.host_ip,
                               checkpoint_transport=transport, timeout=timedelta(seconds=a.communication_timeout),
                               world_size_mode=(WorldSizeMode.FIXED_WITH_SPARES
                                                if a.world_size_mode == "fixed_with_spares"
                                                else WorldSizeMode.DYNAMIC), event=self.event)
        snap = _Snapshot(st, self.device) if a.snapshot_overlap else None
        state_bytes = st.numel * (st.param[0].element_size() + 3 * 4)
        self.event("ready", probe=True, numel=st.numel, state_bytes=state_bytes, device=str(self.device),
                   hashes=self.current_hashes() if a.audit_state else {})
        deadline = time.monotonic() + a.max_seconds
        while not self.marker("START").exists():
            if self.marker("STOP").exists() or time.monotonic() > deadline:
                raise RuntimeError("Stopped or timed out before START")
            time.sleep(0.02)
        mgr = self.manager
        while not self.requested_stop() and time.monotonic() < deadline and self.progress["updates"] < a.steps:
            t0 = time.monotonic()
            self.boundary_rng = dict(step=self.progress["updates"], rng=self.rng_snapshot())
            mgr.start_quorum()
            step = self.progress["updates"]
            t1 = time.monotonic()
            src = snap.begin() if snap is not None else None
            st.grad.copy_(self.gradient(step))
            mgr.allreduce(st.grad).wait()
            if self.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
            t2 = time.monotonic()
            self.engine.optimizer_step([st.grad], 1.0)
            if self.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
            t3 = time.monotonic()
            if snap is not None:
                self.event("snapshot_overlap", step=step, **snap.finish(src))
            if mgr.should_commit():
                self.engine.commit()
                self.progress["updates"] += 1
                self.event("commit", step=self.progress["updates"], participants=mgr.num_participants(),
                           contributed=mgr.is_participating(),
                           quorum_seconds=t1 - t0, reduce_seconds=t2 - t1, optimizer_seconds=t3 - t2,
                           seconds=time.monotonic() - t0,
                           hashes=self.current_hashes() if (a.hash_every and a.audit_state) else {})
            else:
                self.event("skipped", step=step, error=str(mgr.errored()))
        self.event("stopped", step=self.progress["updates"])
        mgr.shutdown()
        self.event.close()


def main(argv=None):
    ProbeWorker(parse_args(argv)).run()


if __name__ == "__main__":
    main()
