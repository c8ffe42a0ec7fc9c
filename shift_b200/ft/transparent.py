"""Transparent mode: an unmodified PyTorch training script under the
fault-tolerance harness.

    python -m shift_b200.ft.transparent --session S --replica R --lighthouse HOST:PORT \
        [--root RESULTS] [--generation G] [--target-steps N] --script train.py [--device cpu|cuda] \
        -- <the script's own arguments>

(as a supervisor entry module: ``"entry_module": "shift_b200.ft.transparent"``
and ``train_args`` starting with ``--script``).  The script runs as
``__main__``, unchanged.  What it does to its optimizers is intercepted on
every ``torch.optim.Optimizer`` it creates:

* ``optimizer.zero_grad()`` begins a step: the replica's Manager takes the
  step's quorum, and a replica that is behind the quorum (a relaunched one)
  first loads a live peer's state -- every parameter the optimizer owns,
  the optimizer's state, the step count and the RNG -- through the packed
  transport, with a SHA-256 audit of what it received;
* ``optimizer.step()`` averages the parameters' gradients over the quorum's
  participants (a healing replica contributes zeros), reports non-finite
  gradients as an error, and runs the real update only if every replica
  votes to commit; otherwise the step is skipped, so a failed vote costs
  nothing to undo.

Between steps the harness honours the session's STOP marker and
``--target-steps`` by raising ``SystemExit`` from ``zero_grad``, and it
writes the same JSONL events as the native trainer (``ready``, ``begin``,
``commit``, ``skipped``, ``restored``, ``stopped``).  The script can read
``SHIFT_REPLICA_ID`` / ``SHIFT_NUM_REPLICAS_HINT`` to shard its own data.

The reference does the same for one specific FLASH script, bound to its
SHA-256 (shift_full/runtime_patch.py:181-354, shift_full/launch.py:25-106):
it wraps that script's optimizer into a commit-gated proxy and moves the
quorum to ``zero_grad`` (:559).  Here any script that uses
``torch.optim`` optimizers is covered, with no patch list.
"""
from __future__ import annotations

import argparse
import os
import random
import runpy
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch

from ..utils.digest import digest
from ..utils.events import EventLog


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--session", required=True)
    p.add_argument("--replica", type=int, required=True)
    p.add_argument("--generation", type=int, default=0)
    p.add_argument("--host-ip", default="127.0.0.1")
    p.add_argument("--root", default="results")
    p.add_argument("--lighthouse", required=True)
    p.add_argument("--min-replicas", type=int, default=1)
    p.add_argument("--target-steps", type=int, default=1_000_000)
    p.add_argument("--device", choices=["cpu", "cuda"], default="cpu")
    p.add_argument("--communication-timeout", type=float, default=30)
    p.add_argument("--max-seconds", type=float, default=900)
    p.add_argument("--script", required=True)
    p.add_argument("script_args", nargs=argparse.REMAINDER)
    a = p.parse_args(argv)
    a.script_args = a.script_args[1:] if a.script_args and a.script_args[0] == "--" else a.script_args
    return a


class TransparentRuntime:
    """The harness around one replica process running a user script."""

    def __init__(self, args):
        self.args = args
        self.out = Path(os.environ.get("SHIFT_RESULT_DIR", str(Path(args.root) / args.session)))
        self.out.mkdir(parents=True, exist_ok=True)
        self.rank = int(os.environ.get("LOCAL_RANK", "0"))
        self.event = EventLog(self.out / f"events_g{args.generation}_r{self.rank}.jsonl", rid=args.replica,
                              rank=self.rank, generation=args.generation, host_ip=args.host_ip)
        self.event.keep = False
        self.device = torch.device("cuda", int(os.environ.get("SHIFT_CUDA_DEVICE", self.rank))) \
            if args.device == "cuda" else torch.device("cpu")
        self.progress = {"updates": 0}
        self.optimizers: list = []
        self.manager = None
        self.in_step = False
        self.step_started = 0.0
        self.started = False

    # ------------------------------------------------------------------ the script's optimizers
    def install(self):
        rt = self
        orig_init = torch.optim.Optimizer.__init__

        def init(opt, *a, **k):
            orig_init(opt, *a, **k)
            rt.adopt(opt)

        torch.optim.Optimizer.__init__ = init
        self._orig_init = orig_init

    def uninstall(self):
        torch.optim.Optimizer.__init__ = self._orig_init

    def adopt(self, opt):
        if getattr(opt, "_shift_adopted", False):
            return
        opt._shift_adopted = True
        self.optimizers.append(opt)
        real_step, real_zero = opt.step, opt.zero_grad

        def zero_grad(*a, **k):
            self.begin_step()
            return real_zero(*a, **k)

        def step(*a, **k):
            return self.gated_step(real_step, a, k)

        opt.zero_grad, opt.step = zero_grad, step

    def params(self) -> list:
        seen, out = set(), []
        for opt in self.optimizers:
            for g in opt.param_groups:
                for p in g["params"]:
                    if id(p) not in seen:
                        seen.add(id(p))
                        out.append(p)
        return out

    # ------------------------------------------------------------------ state for heal
    def export_state(self):
        return {"params": [p.detach() for p in self.params()],
                "optimizers": [o.state_dict() for o in self.optimizers], "progress": dict(self.progress),
                "torch_rng": torch.get_rng_state(), "python_rng": random.getstate(),
                "step": self.progress["updates"], "source_replica": self.args.replica, "source_rank": self.rank,
                "hashes": self.hashes()}

    def load_state(self, payload):
        t0 = time.monotonic()
        assert payload["source_rank"] == self.rank and payload["step"] == payload["progress"]["updates"]
        with torch.no_grad():
            for p, src in zip(self.params(), payload["params"]):
                p.copy_(src)
        for o, sd in zip(self.optimizers, payload["optimizers"]):
            o.load_state_dict(sd)
        self.progress.update(payload["progress"])
        torch.set_rng_state(payload["torch_rng"])
        random.setstate(payload["python_rng"])
        ok = self.hashes() == payload["hashes"]
        self.event("restored", step=payload["step"], load_seconds=time.monotonic() - t0, hashes_match=ok,
                   source_replica=payload["source_replica"], source_rank=payload["source_rank"],
                   optimizer_tensors=sum(len(sd.get("state", {})) for sd in payload["optimizers"]))
        assert ok, "restored state differs from the donor's snapshot"

    def hashes(self) -> dict:
        return {"model": digest([p.detach().cpu() for p in self.params()]),
                "optimizer": digest([o.state_dict() for o in self.optimizers]), "progress": digest(self.progress)}

    # ------------------------------------------------------------------ per step
    def ensure_manager(self):
        if self.manager is not None:
            return self.manager
        from .manager import Manager
        from .process_group import ReconfigurableGroup
        from .train import _free_port
        from .transport import PackedTransport
        a = self.args
        backend = "nccl" if self.device.type == "cuda" else "gloo"
        pg = ReconfigurableGroup(backend, a.communication_timeout, self.device if backend == "nccl" else None,
                                 prefix=f"t{self.rank}", event=self.event)
        transport = PackedTransport(pg, self.device if backend == "nccl" else torch.device("cpu"),
                                    timedelta(seconds=a.communication_timeout), self.event)
        store_port = int(os.environ.get("SHIFT_STORE_PORT", "0")) or _free_port()
        self.manager = Manager(pg, self.load_state, self.export_state, a.min_replicas, f"shift{a.replica}",
                               a.lighthouse, rank=self.rank, world_size=1, store_addr=f"{a.host_ip}:{store_port}",
                               hostname=a.host_ip, checkpoint_transport=transport,
                               timeout=timedelta(seconds=a.communication_timeout), event=self.event)
        self.event("ready", mode="transparent", script=a.script, params=sum(p.numel() for p in self.params()),
                   hashes=self.hashes())
        deadline = time.monotonic() + a.max_seconds
        while not (self.out / "START").exists():
            if (self.out / "STOP").exists() or time.monotonic() > deadline:
                raise RuntimeError("stopped or timed out before START")
            time.sleep(0.02)
        return self.manager

    def stop_requested(self) -> bool:
        m = self.out / "STOP"
        if self.progress["updates"] >= self.args.target_steps:
            return True
        if not m.exists():
            return False
        text = m.read_text().strip()
        return not text or self.progress["updates"] >= int(text)

    def begin_step(self):
        if self.in_step:                    # zero_grad called again within one step
            return
        mgr = self.ensure_manager()
        if self.stop_requested():
            self.finish()
            raise SystemExit(0)
        self.step_started = time.monotonic()
        if self.args.generation > 0 and not self.started:
            self.event("recovery_request", step=self.progress["updates"])
        self.started = True
        mgr.start_quorum()
        self.in_step = True
        self.event("begin", step=self.progress["updates"], participants=mgr.num_participants())

    def gated_step(self, real_step, a, k):
        if not self.in_step:
            self.begin_step()
        mgr = self.manager
        grads = [p.grad for p in self.params() if p.grad is not None]
        if grads:
            flat = torch.cat([g.reshape(-1).float() for g in grads])
            mgr.allreduce(flat).wait()
            if not bool(torch.isfinite(flat).all()):
                mgr.report_error(RuntimeError("non-finite gradients"))
            off = 0
            for g in grads:
                g.copy_(flat[off:off + g.numel()].view_as(g).to(g.dtype))
                off += g.numel()
        ret = None
        if mgr.should_commit():
            ret = real_step(*a, **k)
            self.progress["updates"] += 1
            self.event("commit", step=self.progress["updates"], participants=mgr.num_participants(),
                       contributed=mgr.is_participating(), hashes=self.hashes(),
                       seconds=time.monotonic() - self.step_started)
        else:
            self.event("skipped", step=self.progress["updates"], error=str(mgr.errored()))
        self.in_step = False
        return ret

    def finish(self):
        self.event("stopped", step=self.progress["updates"])
        if self.manager is not None:
            self.manager.shutdown()
        self.event.close()

    # ------------------------------------------------------------------ main
    def run(self):
        a = self.args
        os.environ["SHIFT_REPLICA_ID"] = str(a.replica)
        os.environ["SHIFT_NUM_REPLICAS_HINT"] = str(max(1, a.min_replicas))
        self.install()
        sys.argv = [a.script, *a.script_args]
        try:
            runpy.run_path(a.script, run_name="__main__")
        except SystemExit as e:
            if e.code not in (None, 0):
                raise
            return
        finally:
            self.uninstall()
        self.finish()                       # the script ended on its own


def main(argv=None):
    TransparentRuntime(parse_args(argv)).run()


if __name__ == "__main__":
    main()
