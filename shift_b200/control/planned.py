"""In-box controller for planned handoff experiments (P1f / P2, rotation cycles).

    python -m shift_b200.control.planned --root results --name S --variant p1f|p2 \
        [--scenario healthy|prepare-fail|ready-timeout|stale-state|relay-reject|slow-compute] \
        [--post-steps 50] [--cancel] [--model tiny|bench] [--device cpu|cuda] [--nproc 1]

Flow (scripts/run_planned_handoff.py of the reference, on one box): start the
coordination store and the epoch-0 lighthouse; launch A and B; START; after
two steps send REQUEST, launch the spare C and the next-epoch lighthouse(s);
when every C rank is prepared, ARM; A's rank 0 selects the cut; wait for
``post_steps`` committed AC steps; write ``planned_summary.json`` with the
handoff interval (last AB commit -> first AC commit on A rank 0) and the
audit checks.
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import subprocess as sp
import sys
import time
from datetime import timedelta
from pathlib import Path

import torch.distributed as dist

from ..ft.native import spawn_lighthouse
from ..utils.events import EventLog, atomic_write
from .event_reader import IncrementalReader


def free_ports(n: int) -> list[int]:
    socks, out = [], []
    for _ in range(n):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        socks.append(s)
        out.append(s.getsockname()[1])
    for s in socks:
        s.close()
    return out


def free_block(size: int = 64) -> int:
    """A base port with ``size`` consecutive free ports above it."""
    for _ in range(200):
        base = free_ports(1)[0]
        if base + size >= 65000:
            continue
        ok = True
        for p in range(base, base + size):
            s = socket.socket()
            try:
                s.bind(("127.0.0.1", p))
            except OSError:
                ok = False
            finally:
                s.close()
            if not ok:
                break
        if ok:
            return base
    raise OSError("no free port block")


class PlannedSession:
    def __init__(self, root, name, variant="p1f", scenario="healthy", model="tiny", device="cpu", nproc=1,
                 audit=True, train_args=None, devices=None, seconds=600, module="shift_b200.ft.planned_train"):
        self.dir = Path(root) / name
        self.dir.mkdir(parents=True, exist_ok=True)
        self.root, self.name = Path(root), name
        self.variant, self.scenario = variant, scenario
        self.model, self.device, self.nproc = model, device, nproc
        self.devices = devices or {}
        self.seconds = seconds
        self.module = module
        self.log = EventLog(self.dir / "controller.jsonl", role="controller")
        self.reader = IncrementalReader(self.dir)
        base = free_block(200)
        self.lh_port = base
        self.coord_port = base + 50
        self.store_base = base + 60
        self.master_base = base + 150
        self.coord = dist.TCPStore("127.0.0.1", self.coord_port, None, True, timeout=timedelta(seconds=60),
                                   wait_for_workers=False)
        self.lighthouses = []
        self.procs: dict[str, sp.Popen] = {}
        args = ["--model", model, "--device", device, "--seq-len", "128", "--batch", "2", "--data", "random",
                "--communication-timeout", "60", "--planned-variant", variant, "--coord",
                f"127.0.0.1:{self.coord_port}", "--steps", "100000"]
        if audit:
            args += ["--audit-state", "--hash-every", "1"]
        if scenario != "healthy":
            args += ["--planned-inject", scenario]
        self.train_args = args + list(train_args or [])

    # ------------------------------------------------------------------ plumbing
    def key(self, k, v="1"):
        self.coord.set(k, str(v))
        self.log("key", key=k, value=str(v))

    def rows(self, kind=None, **m):
        self.reader.poll()
        return self.reader.rows(kind, **m)

    def wait(self, label, pred, timeout=300):
        end = time.monotonic() + timeout
        while time.monotonic() < end:
            self.reader.poll()
            v = pred()
            if v:
                self.log(label)
                return v
            for role, p in self.procs.items():
                if p.poll() not in (None, 0):
                    raise RuntimeError(f"role {role} exited with {p.returncode} while waiting for {label}")
            time.sleep(0.02)
        raise TimeoutError(label)

    def start_lighthouse(self, slot, min_replicas=2):
        """Start the lighthouse of one epoch (``slot`` = 10 * epoch, + 1 for the
        fallback A+B epoch of a P2 round) on a port the OS chooses, and publish
        its address under ``lighthouse/<slot>`` of the coordination store,
        where the trainers look it up: no fixed port that another process may
        have taken in the meantime."""
        p, addr = spawn_lighthouse("127.0.0.1:0", min_replicas=min_replicas, join_timeout_ms=1000,
                                   heartbeat_timeout_ms=1000, quorum_tick_ms=20)
        self.lighthouses.append(p)
        self.coord.set(f"lighthouse/{slot}", addr)
        self.log("lighthouse_started", slot=slot, address=addr)

    def launch(self, role: str, name: str | None = None, generation: int | None = None, round_: int = 0,
               extra=()):
        """Launch one replica process tree.  ``name`` is the physical process
        (A, B or C; in a rotation the spare alternates between C and B);
        ``role`` its protocol role at launch."""
        name = name or role
        rid = 0 if role == "A" else 1
        gen = (1 if role == "C" else 0) if generation is None else generation
        env = dict(os.environ)
        env["PYTHONPATH"] = str(Path(__file__).resolve().parents[2]) + os.pathsep + env.get("PYTHONPATH", "")
        env["SHIFT_RESULT_DIR"] = str(self.dir)
        env["SHIFT_STORE_PORT"] = str(self.store_base + 20 * {"A": 0, "B": 1, "C": 2}[name])
        env.setdefault("NCCL_NVLS_ENABLE", "0")
        cmd = [sys.executable, "-m", "shift_b200.control.launch", "--nproc", str(self.nproc), "--master-port",
               str(self.master_base + 10 * {"A": 0, "B": 1, "C": 2}[name]), "--module", self.module]
        if name in self.devices:
            cmd += ["--devices", ",".join(str(d) for d in self.devices[name])]
        cmd += ["--", "--session", self.name, "--replica", str(rid), "--generation", str(gen), "--root",
                str(self.root), "--planned-role", role, "--planned-round", str(round_), *self.train_args, *extra]
        log = (self.dir / f"role_{name}_g{gen}.log").open("w")
        self.procs[name] = sp.Popen(cmd, env=env, stdout=log, stderr=sp.STDOUT)
        self.log("launched", role=role, name=name, generation=gen, round=round_, pid=self.procs[name].pid)

    def commits(self, rid, gen, rank=0):
        return self.reader.rows("commit", rid=rid, generation=gen, rank=rank)

    # ------------------------------------------------------------------ experiment
    def run(self, post_steps=3, cancel=False):
        n = self.nproc
        self.start_lighthouse(0)
        self.launch("A")
        self.launch("B")
        self.wait("ab_ready", lambda: len(self.rows("ready", generation=0)) == 2 * n, 300)
        atomic_write(self.dir / "START", "")
        self.wait("ab_two_steps", lambda: all(any(c["step"] >= 2 for c in self.commits(r, 0)) for r in (0, 1)))
        t_request = time.time()
        self.log("REQUEST", variant=self.variant)
        self.launch("C")
        self.key("request")
        self.start_lighthouse(10)
        if self.variant == "p2":
            self.start_lighthouse(11)
        if self.scenario in ("prepare-fail", "ready-timeout") or cancel:
            kind = {"prepare-fail": "planned_prepare_rejected", "ready-timeout": "planned_prepare_delayed"}.get(
                self.scenario, "planned_local_ready")
            self.wait("c_state", lambda: len(self.rows(kind, generation=1)) == n)
            latest = max(c["step"] for c in self.commits(0, 0))
            until = latest + 4
            atomic_write(self.dir / "TRAIN_UNTIL", str(until))
            self.key("cancel", self.scenario if self.scenario != "healthy" else "1")
            self.wait("all_cancelled", lambda: len(self.rows("planned_cancelled")) >= 3 * n)
            self.wait("ab_continue", lambda: all(any(c["step"] >= until for c in self.commits(r, 0)) for r in (0, 1)))
            return self.finish({"cancelled": True, "scenario": self.scenario, "final_step": until})
        self.wait("c_local_ready", lambda: len(self.rows("planned_local_ready", generation=1)) == n)
        self.key("arm")
        cut = self.wait("cut_selected", lambda: self.rows("planned_cut_selected", rid=0))[-1]["step"]
        target = cut + post_steps
        atomic_write(self.dir / "TRAIN_UNTIL", str(target))
        if self.scenario == "relay-reject" or self.scenario == "stale-state":
            self.wait("ab_recovered_or_cancelled",
                      lambda: self.rows("planned_new_epoch_ab_recovered") or len(self.rows("planned_cancelled")) >= n,
                      300)
            self.wait("ab_target", lambda: any(c["step"] >= target for c in self.commits(0, 0)), 300)
        else:
            self.wait("ac_target", lambda: any(c["step"] >= target for c in self.commits(1, 1)), 600)
        return self.finish({"cut": cut, "t_request": t_request, "post_steps": post_steps})

    def run_cycles(self, cycles=3, post_steps=6):
        """Continuous B/C rotation: ``cycles`` consecutive planned handoffs.
        Round r hands replica 1 from the process that won round r-1 (or B) to
        a freshly launched spare (physical C in even rounds, a relaunched B in
        odd ones), epoch r -> r+1; ``post_steps`` committed steps follow each
        cut before the next request."""
        n = self.nproc
        extra = ["--planned-cycles", str(cycles)]
        self.start_lighthouse(0)
        self.launch("A", extra=extra)
        self.launch("B", extra=extra)
        self.wait("ab_ready", lambda: len(self.rows("ready", generation=0)) == 2 * n, 300)
        atomic_write(self.dir / "START", "")
        self.wait("ab_two_steps", lambda: all(any(c["step"] >= 2 for c in self.commits(r, 0)) for r in (0, 1)))
        cuts, t_requests = [], []
        for r in range(cycles):
            spare = "C" if r % 2 == 0 else "B"
            if spare in self.procs:                         # the previous owner of that name has retired
                self.wait(f"retired_{spare}_{r}", lambda: self.procs[spare].poll() is not None, 300)
            pre = f"round/{r}/" if r else ""
            t_requests.append(time.time())
            self.log("REQUEST", variant=self.variant, round=r)
            self.launch("C", name=spare, generation=r + 1, round_=r, extra=extra)
            self.key(pre + "request")
            self.start_lighthouse(10 * (r + 1))
            if self.variant == "p2":
                self.start_lighthouse(10 * (r + 1) + 1)
            self.wait(f"c_local_ready_{r}", lambda: len(self.rows("planned_local_ready", generation=r + 1)) == n)
            self.key(pre + "arm")
            cut = self.wait(f"cut_selected_{r}", lambda: [x for x in self.rows("planned_cut_selected", rid=0)
                                                         if x.get("round", 0) == r])[-1]["step"]
            cuts.append(cut)
            target = cut + post_steps
            if r == cycles - 1:
                atomic_write(self.dir / "TRAIN_UNTIL", str(target))
            self.wait(f"post_steps_{r}", lambda: any(c["step"] >= target for c in self.commits(0, 0)), 600)
        return self.finish({"cuts": cuts, "t_requests": t_requests, "post_steps": post_steps, "cycles": cycles})

    def finish(self, info):
        atomic_write(self.dir / "STOP", "")
        for role, p in self.procs.items():
            try:
                p.wait(120)
            except sp.TimeoutExpired:
                p.kill()
        for p in self.lighthouses:
            p.terminate()
            p.wait(10)
        self.reader.poll()
        summary = summarize(self.reader, self.variant, info, self.nproc)
        summary["returncodes"] = {r: p.returncode for r, p in self.procs.items()}
        (self.dir / "planned_summary.json").write_text(json.dumps(summary, indent=1, sort_keys=True, default=str))
        self.log.close()
        return summary


def summarize_cycles(reader, variant, info, nproc=1) -> dict:
    """Per-round handoff interval, exposed transfer time and audits of a rotation."""
    rows = reader.all_rows
    a0 = sorted((r for r in rows if r["kind"] == "commit" and r["rid"] == 0 and r["rank"] == 0),
                key=lambda r: r["step"])
    by_step = {r["step"]: r for r in a0}
    cuts = info["cuts"]
    normal = [b["time"] - a["time"] for a, b in zip(a0, a0[1:])
              if b["step"] == a["step"] + 1 and all(not (c <= a["step"] <= c + 1) for c in cuts)]
    med = sorted(normal)[len(normal) // 2] if normal else 0.0
    out = {"variant": variant, **info, "normal_step_s": med, "rounds": []}
    checks = {}
    for r, cut in enumerate(cuts):
        gen = r + 1
        rd = {"round": r, "cut": cut}
        if cut in by_step and cut + 1 in by_step:
            rd["handoff_interval_s"] = by_step[cut + 1]["time"] - by_step[cut]["time"]
            rd["exposed_transfer_s"] = rd["handoff_interval_s"] - med
        recv = [x for x in rows if x["kind"] == "commit" and x["rid"] == 1 and x["generation"] == gen]
        exact, compared = True, 0
        for c in recv:
            a = next((x for x in a0 if x["step"] == c["step"] and x["rank"] == c["rank"]), None)
            if a and a.get("hashes") and c.get("hashes"):
                compared += 1
                for k in ("model", "optimizer", "scheduler"):
                    exact &= a["hashes"].get(k) == c["hashes"].get(k)
        restored = [x for x in rows if x["kind"] == "restored" and x["generation"] == gen]
        rd["compared_commits"] = compared
        checks[f"round{r}_state_exact"] = {"pass": exact and compared > 0, "compared": compared}
        checks[f"round{r}_restore_hashes_match"] = {"pass": bool(restored) and all(x["hashes_match"]
                                                                                  for x in restored)}
        if variant == "p2":
            rel = [x for x in rows if x["kind"] == "planned_gradient_received" and x["generation"] == gen]
            checks[f"round{r}_gradient_relay"] = {"pass": len(rel) >= nproc and all(
                x.get("forward_calls") == 0 for x in rel)}
        out["rounds"].append(rd)
    checks["monotonic_a"] = {"pass": all(b["step"] == a["step"] + 1 for a, b in zip(a0, a0[1:]))}
    out["checks"] = checks
    out["pass"] = all(c["pass"] for c in checks.values())
    return out


def summarize(reader, variant, info, nproc=1) -> dict:
    """Handoff interval and audit checks from a session's events."""
    if "cuts" in info:
        return summarize_cycles(reader, variant, info, nproc)
    rows = reader.all_rows
    a0 = [r for r in rows if r["kind"] == "commit" and r["rid"] == 0 and r["rank"] == 0 and r["generation"] == 0]
    checks = {}
    out = {"variant": variant, **info}
    cut = info.get("cut")
    if cut is None:
        out["checks"] = {"cancel_kept_old_epoch": {"pass": all(r.get("epoch", 0) == 0 for r in a0)}}
        out["pass"] = all(c["pass"] for c in out["checks"].values())
        return out
    last_ab = [r for r in a0 if r["step"] == cut]
    first_new = [r for r in a0 if r["step"] == cut + 1]
    if last_ab and first_new:
        normal = [b["time"] - a["time"] for a, b in zip(a0, a0[1:]) if b["step"] < cut]
        med = sorted(normal)[len(normal) // 2] if normal else 0.0
        out["handoff_interval_s"] = first_new[0]["time"] - last_ab[0]["time"]
        out["normal_step_s"] = med
        out["extra_interval_s"] = out["handoff_interval_s"] - med
        out["request_to_first_new_commit_s"] = first_new[0]["time"] - info.get("t_request", first_new[0]["time"])
    c_commits = [r for r in rows if r["kind"] == "commit" and r["rid"] == 1 and r["generation"] == 1]
    a_after = {(r["step"], r["rank"]): r for r in rows if r["kind"] == "commit" and r["rid"] == 0 and r["step"] > cut}
    exact, compared = True, 0
    for c in c_commits:
        a = a_after.get((c["step"], c["rank"]))
        if a and a.get("hashes") and c.get("hashes"):
            compared += 1
            for k in ("model", "optimizer", "scheduler"):
                exact &= a["hashes"].get(k) == c["hashes"].get(k)
    recovered = [r for r in rows if r["kind"] == "planned_new_epoch_ab_recovered"]
    # a handoff called off at the cut (the spare rejected a stale pre-copied
    # state): every process reports the cancellation and A keeps committing in
    # the old epoch past the cut
    cancelled = [r for r in rows if r["kind"] == "planned_cancelled" and r.get("step") == cut]
    if recovered:
        checks["ab_recovered_new_epoch"] = {"pass": all(r.get("old_manager_rejected") for r in recovered)}
        checks["c_effective_commits_zero"] = {"pass": not c_commits}
    elif cancelled:
        after = [r for r in a0 if r["step"] > cut]
        checks["cancelled_at_cut"] = {"pass": len(cancelled) >= 3 * nproc, "reports": len(cancelled)}
        checks["old_epoch_kept"] = {"pass": bool(after) and all(r.get("epoch", 0) == 0 for r in after)}
        checks["c_effective_commits_zero"] = {"pass": not c_commits}
        rejected = [r for r in rows if r["kind"] == "planned_precopy_rejected"]
        if rejected:
            checks["stale_state_rejected"] = {"pass": True, "reports": len(rejected)}
    else:
        checks["ac_state_exact"] = {"pass": exact and compared > 0, "compared": compared}
        checks["no_b_in_ac"] = {"pass": all("B" not in r.get("physical_members", []) for r in c_commits)}
        checks["epoch_activated"] = {"pass": all(r.get("epoch", 0) >= 1 for r in c_commits) and bool(c_commits)}
        b_rej = [r for r in rows if r["kind"] == "planned_old_commit_rejected"]
        checks["retired_b_rejected"] = {"pass": len(b_rej) >= nproc}
        restored = [r for r in rows if r["kind"] == "restored" and r["generation"] == 1]
        checks["restore_hashes_match"] = {"pass": bool(restored) and all(r["hashes_match"] for r in restored)}
        if variant == "p2":
            rel = [r for r in rows if r["kind"] == "planned_gradient_received"]
            checks["gradient_relay_exact"] = {"pass": len(rel) >= nproc}
            checks["c_no_relay_forward"] = {"pass": all(r.get("forward_calls") == 0 for r in rel) and bool(rel)}
            relay_commit = [r for r in c_commits if r.get("relay_step")]
            checks["relay_step_committed_by_c"] = {"pass": bool(relay_commit) and all(
                r.get("forward_calls", 1) == 0 for r in relay_commit)}
    checks["monotonic_a"] = {"pass": all(b["step"] == a["step"] + 1 for a, b in zip(a0, a0[1:]))}
    out["checks"] = checks
    out["pass"] = all(c["pass"] for c in checks.values())
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--root", default="results")
    ap.add_argument("--name", required=True)
    ap.add_argument("--variant", choices=["p1f", "p2"], default="p1f")
    ap.add_argument("--scenario", default="healthy",
                    choices=["healthy", "prepare-fail", "ready-timeout", "stale-state", "relay-reject", "slow-compute"])
    ap.add_argument("--post-steps", type=int, default=3)
    ap.add_argument("--cancel", action="store_true")
    ap.add_argument("--cycles", type=int, default=1, help="consecutive B/C rotation rounds (1 = one handoff)")
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--nproc", type=int, default=1)
    ap.add_argument("--gpus", default="", help="A,B,C device lists, e.g. '0;1;2'")
    ap.add_argument("--train-args", default="", help="extra trainer flags, e.g. '--seq-len 2048 --batch 4'")
    ap.add_argument("--module", default="shift_b200.ft.planned_train",
                    help="worker module; shift_b200.ft.mp_planned_train hands over TP x PP replicas "
                         "(--nproc tp*pp, --train-args '--tp 2 --pp 2 ...')")
    ap.add_argument("--runs", type=int, default=1, help="independent handoff sessions (name_1, name_2, ...)")
    ap.add_argument("--no-preflight", action="store_true",
                    help="skip the check that no other compute process holds the session's GPUs")
    a = ap.parse_args(argv)
    devices = {}
    if a.gpus:
        for role, lst in zip("ABC", a.gpus.split(";")):
            devices[role] = [int(x) for x in lst.split(",")]
    if a.device == "cuda":
        # A reduces with B, then with C, inside kernels that wait on the other
        # role's flags: A never shares a GPU with either.  B and C are never in
        # one quorum (C replaces B), so they may share GPUs.
        clash = set(devices.get("A", [])) & (set(devices.get("B", [])) | set(devices.get("C", [])))
        if clash:
            raise SystemExit(f"GPUs {sorted(clash)} are given to role A and to role B or C: roles that wait on "
                             "each other inside kernels must not share a GPU")
    if a.device == "cuda" and not a.no_preflight:
        from .preflight import check_gpus_idle
        wanted = sorted({g for lst in devices.values() for g in lst}) or None
        pre = check_gpus_idle(wanted)
        if not pre["pass"]:
            print(json.dumps({"pass": False, "preflight": pre}, default=str))
            return 2
    import shlex
    results = []
    for i in range(a.runs):
        name = a.name if a.runs == 1 else f"{a.name}_{i + 1}"
        s = PlannedSession(a.root, name, a.variant, a.scenario, a.model, a.device, a.nproc, devices=devices,
                           train_args=shlex.split(a.train_args), module=a.module)
        res = s.run_cycles(a.cycles, a.post_steps) if a.cycles > 1 else s.run(a.post_steps, a.cancel)
        print(json.dumps({k: v for k, v in res.items() if k != "checks"}, indent=1, default=str))
        print(json.dumps({k: v["pass"] for k, v in res.get("checks", {}).items()}, indent=1))
        results.append(res)
    if a.runs > 1:
        ivs = sorted(r["handoff_interval_s"] for r in results if r.get("handoff_interval_s") is not None)
        agg = {"runs": a.runs, "variant": a.variant, "module": a.module, "intervals_s": ivs,
               "median_interval_s": ivs[len(ivs) // 2] if ivs else None,
               "all_pass": all(r.get("pass") for r in results)}
        (Path(a.root) / f"{a.name}_runs.json").write_text(json.dumps(agg, indent=1) + "\n")
        print(json.dumps(agg, indent=1))
    return 0 if all(r.get("pass") for r in results) else 1


if __name__ == "__main__":
    raise SystemExit(main())
