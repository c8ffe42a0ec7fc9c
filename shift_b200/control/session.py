"""In-box cluster controller (the reference's laptop-side ``Session`` without
ssh / docker: every replica's supervisor is a local process).

    python -m shift_b200.control.session --config cfg.json --session S \
        [--replicas 2] [--faults N] [--fault-step K] [--interval SEC] [--worker-kill RANK]

``Session.start`` launches one supervisor per replica, waits until every rank
of every replica reported ``ready``, then writes START (shift_full/control.py:265-281).
A fault writes ``KILL_g<G>_r<R>`` (or WORKER_KILL), waits for the survivor to
commit solo, requests ``RESTART_g<G+1>_r<R>``, waits for every relaunched rank
to be ``restored`` and for ``joint`` commits past the restored step
(shift_full/control.py:307-339).  Evidence stays in ``<root>/<session>``.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess as sp
import sys
import time
from pathlib import Path

from ..utils.events import EventLog, atomic_write
from .event_reader import IncrementalReader
from .supervisor import load_config


def joint_boundary(commits, rid, gen, after_step, replicas, ranks):
    """First joint commit of replica ``rid`` (generation ``gen``) past
    ``after_step``: the smallest step at which EVERY rank of the replica
    committed with all ``replicas`` participating and itself contributing
    (a commit the replica made while healing, without contributing its
    gradient, does not count).  Returns (step, latest commit time over the
    ranks) or None.  The rule of the reference's rotation boundary
    (sf/rotation.py; sf/test_rotation.py:9-43)."""
    per_step: dict = {}
    for c in commits:
        if (c.get("kind", "commit") != "commit" or c.get("rid") != rid or c.get("generation", 0) != gen
                or c.get("step", 0) <= after_step or c.get("participants") != replicas
                or c.get("contributed") is False):
            continue
        per_step.setdefault(c["step"], {})[c.get("rank", 0)] = c.get("time")
    for step in sorted(per_step):
        got = per_step[step]
        if all(r in got for r in range(ranks)):
            return step, max(t for t in got.values() if t is not None)
    return None


class Session:
    def __init__(self, root, session: str, config_path, replicas: int = 2, host_ip: str = "127.0.0.1",
                 seconds: float = 900.0):
        self.root = Path(root)
        self.session = session
        self.dir = self.root / session
        self.dir.mkdir(parents=True, exist_ok=True)
        self.config_path = str(config_path)
        self.cfg = load_config(config_path)
        self.replicas = replicas
        self.host_ip = host_ip
        self.seconds = seconds
        self.reader = IncrementalReader(self.dir)
        self.sup: dict[int, sp.Popen] = {}
        self.generation = {r: 0 for r in range(replicas)}
        self.log = EventLog(self.dir / "controller.jsonl", role="controller")
        self.timings: list[dict] = []

    # ------------------------------------------------------------------ plumbing
    def marker(self, name: str, text: str = ""):
        atomic_write(self.dir / name, text)
        self.log("marker", name=name, text=text)

    def poll(self):
        self.reader.poll()

    def rows(self, kind=None, **m):
        self.poll()
        return self.reader.rows(kind, **m)

    def await_(self, pred, timeout: float, what: str, interval: float = 0.02):
        t0 = time.monotonic()
        while True:
            self.poll()
            v = pred()
            if v:
                return v
            for r, p in self.sup.items():
                if p.poll() is not None and p.returncode != 0:
                    raise RuntimeError(f"supervisor of replica {r} exited with {p.returncode} while awaiting {what}")
            if time.monotonic() - t0 > timeout:
                raise TimeoutError(f"timed out after {timeout}s awaiting {what}")
            time.sleep(interval)

    def ranks(self) -> int:
        return self.cfg["nproc_per_node"]

    def ready(self, rid, gen):
        return {r["rank"] for r in self.reader.rows("ready", rid=rid, generation=gen)}

    def commits(self, rid, gen=None, rank=0):
        m = dict(rid=rid, rank=rank)
        if gen is not None:
            m["generation"] = gen
        return self.reader.rows("commit", **m)

    def _joint(self, rid, gen, after_step):
        rows = [c for r in range(self.ranks()) for c in self.commits(rid, gen, rank=r)]
        return joint_boundary(rows, rid, gen, after_step, self.replicas, self.ranks())

    def last_step(self, rid, rank=0) -> int:
        c = self.commits(rid, rank=rank)
        return c[-1]["step"] if c else 0

    # ------------------------------------------------------------------ lifecycle
    def start(self, timeout: float = 300.0):
        env = dict(os.environ)
        env["PYTHONPATH"] = str(Path(__file__).resolve().parents[2]) + os.pathsep + env.get("PYTHONPATH", "")
        for r in range(self.replicas):
            cmd = [sys.executable, "-m", "shift_b200.control.supervisor", "--session", self.session, "--replica",
                   str(r), "--root", str(self.root), "--config", self.config_path, "--host-ip", self.host_ip,
                   "--seconds", str(self.seconds)]
            log = (self.dir / f"supervisor_r{r}.log").open("w")
            self.sup[r] = sp.Popen(cmd, env=env, stdout=log, stderr=sp.STDOUT)
            if r == 0 and not self.cfg["external_lighthouse"]:
                self.await_(lambda: self.reader.rows("lighthouse_started"), 60, "lighthouse")
        t0 = time.monotonic()
        self.await_(lambda: all(len(self.ready(r, 0)) == self.ranks() for r in range(self.replicas)), timeout,
                    "all ranks ready")
        self.log("all_ready", seconds=time.monotonic() - t0)
        self.marker("START")

    def fault(self, rid: int, kind: str = "launcher", rank: int = 0, solo_commits: int = 1, timeout: float = 120.0):
        """Kill replica ``rid`` (whole launcher tree, or one rank), wait for the
        survivors to commit solo, restart it, and time the recovery."""
        gen = self.generation[rid]
        survivors = [r for r in range(self.replicas) if r != rid]
        base = {s: self.last_step(s) for s in survivors}
        name = f"KILL_g{gen}_r{rid}" if kind == "launcher" else f"WORKER_KILL_g{gen}_r{rid}"
        t_fault = time.time()
        self.marker(name, str(rank) if kind != "launcher" else "")
        self.await_(lambda: self.reader.rows("injected", rid=rid, generation=gen), 30, "fault injection")
        # survivors continue alone
        self.await_(lambda: all(any(c["participants"] == len(survivors) and c["step"] > base[s]
                                    for c in self.commits(s)[-5:]) for s in survivors) or
                    all(self.last_step(s) >= base[s] + solo_commits for s in survivors), timeout, "solo commits")
        t_solo = time.time()
        self.marker(f"RESTART_g{gen + 1}_r{rid}")
        self.generation[rid] = gen + 1
        self.await_(lambda: len({r["rank"] for r in self.reader.rows("restored", rid=rid, generation=gen + 1)})
                    == self.ranks(), timeout, "restored ranks")
        restored = self.reader.rows("restored", rid=rid, generation=gen + 1)
        rstep = max(r["step"] for r in restored)
        t_restored = max(r["time"] for r in restored)
        # first step every rank of the replica committed jointly past the restored step
        self.await_(lambda: self._joint(rid, gen + 1, rstep) is not None, timeout, "joint commit")
        jstep, jtime = self._joint(rid, gen + 1, rstep)
        joint = {"step": jstep, "time": jtime}
        rec = dict(rid=rid, fault_kind=kind, generation=gen, fault_time=t_fault, solo_time=t_solo,
                   restored_time=t_restored, joint_time=joint["time"], restored_step=rstep, joint_step=joint["step"],
                   fault_to_joint=joint["time"] - t_fault, restored_hashes_match=all(r["hashes_match"] for r in restored))
        self.timings.append(rec)
        self.log("fault_recovered", **rec)
        return rec

    def unplanned_fault(self, rid: int, timeout: float = 300.0):
        """A fault the replica injects into itself (``--inject sigkill_bwd@STEP``
        of the model-parallel worker: one rank SIGKILLs itself mid-backward):
        expect the replica's exit, wait for the survivors' solo commits, restart
        it (on its ``restart_devices``), and time fault -> restored -> first
        joint commit."""
        gen = self.generation[rid]
        survivors = [r for r in range(self.replicas) if r != rid]
        self.marker(f"EXPECT_PEER_FAILURE_g{gen}_r{rid}")
        self.await_(lambda: self.reader.rows("injected_sigkill", rid=rid, generation=gen), timeout, "self-kill")
        kill = self.reader.rows("injected_sigkill", rid=rid, generation=gen)[0]
        base = kill["step"]
        self.await_(lambda: self.reader.rows("peer_fault_exit", rid=rid), timeout, "replica exit")
        self.await_(lambda: all(any(c["participants"] == len(survivors) and c["step"] > base
                                    for c in self.commits(s)) for s in survivors), timeout, "solo commits")
        t_solo = time.time()
        self.marker(f"RESTART_g{gen + 1}_r{rid}")
        self.generation[rid] = gen + 1
        self.await_(lambda: len({r["rank"] for r in self.reader.rows("restored", rid=rid, generation=gen + 1)})
                    == self.ranks(), timeout, "restored ranks")
        restored = self.reader.rows("restored", rid=rid, generation=gen + 1)
        rstep = max(r["step"] for r in restored)
        self.await_(lambda: self._joint(rid, gen + 1, rstep) is not None, timeout, "joint commit")
        jstep, jtime = self._joint(rid, gen + 1, rstep)
        joint = {"step": jstep, "time": jtime}
        placement = {r["rank"]: r.get("placement") for r in self.reader.rows("ready", rid=rid, generation=gen + 1)}
        old_placement = {r["rank"]: r.get("placement") for r in self.reader.rows("ready", rid=rid, generation=gen)}
        ta = self.cfg["train_args"]
        inj = ta[ta.index("--inject") + 1].split("@")[0] if "--inject" in ta else "sigkill_bwd"
        kind = {"sigkill_bwd": "sigkill_mid_backward", "sigkill_step": "sigkill_between_steps"}.get(inj, inj)
        rec = dict(rid=rid, fault_kind=kind, generation=gen, killed_rank=kill["rank"],
                   killed_stage=kill.get("stage"), killed_tp_rank=kill.get("tp_rank"), fault_step=base,
                   fault_time=kill["fault_time"], solo_time=t_solo, restored_time=max(r["time"] for r in restored),
                   joint_time=joint["time"], restored_step=rstep, joint_step=joint["step"],
                   time_to_recovery=joint["time"] - kill["fault_time"],
                   restored_hashes_match=all(r["hashes_match"] for r in restored),
                   placement_before=old_placement, placement_after=placement)
        self.timings.append(rec)
        self.log("fault_recovered", **rec)
        return rec

    def throughput_window(self, rid: int, first_step: int, steps: int = 100) -> dict:
        """Tokens/s of the job per 10-step window from ``first_step`` on, from
        a surviving replica's commits (``tokens`` = tokens of all participants)."""
        rows = sorted((c for c in self.reader.rows("commit", rid=rid, rank=0) if c.get("tokens")),
                      key=lambda c: c["time"])
        rows = [c for c in rows if first_step <= c["step"] <= first_step + steps]
        out = []
        for i in range(0, len(rows) - 10, 10):
            w = rows[i:i + 11]
            dt = w[-1]["time"] - w[0]["time"]
            out.append({"steps": [w[0]["step"], w[-1]["step"]], "tokens_per_s": sum(c["tokens"] for c in w[1:]) / dt,
                        "participants": sorted({c["participants"] for c in w[1:]})})
        return {"windows": out, "steps": len(rows)}

    def finish(self, stop_at_step: int | None = None, timeout: float = 120.0):
        self.marker("STOP", "" if stop_at_step is None else str(stop_at_step))
        for r, p in self.sup.items():
            try:
                p.wait(timeout)
            except sp.TimeoutExpired:
                p.kill()
        self.poll()
        self.log("finished", returncodes={r: p.returncode for r, p in self.sup.items()})
        self.log.close()
        return {r: p.returncode for r, p in self.sup.items()}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    ap.add_argument("--session", required=True)
    ap.add_argument("--root", default="results")
    ap.add_argument("--replicas", type=int, default=2)
    ap.add_argument("--faults", type=int, default=1)
    ap.add_argument("--fault-step", type=int, default=5)
    ap.add_argument("--interval", type=float, default=0.0,
                    help="seconds to keep training between a recovery and the next fault (on top of --fault-step)")
    ap.add_argument("--victim", type=int, default=1)
    ap.add_argument("--worker-kill", type=int, default=None, help="kill one rank instead of the launcher tree")
    ap.add_argument("--joint-commits", type=int, default=3)
    ap.add_argument("--seconds", type=float, default=900)
    ap.add_argument("--unplanned", type=int, default=None,
                    help="replica that injects its own fault (the config's --inject / --inject-rank); "
                         "report time-to-recovery and the tokens/s windows over --window steps")
    ap.add_argument("--window", type=int, default=100)
    a = ap.parse_args(argv)
    s = Session(a.root, a.session, a.config, a.replicas, seconds=a.seconds)
    s.start()
    results = []
    if a.unplanned is not None:
        try:
            survivor = next(r for r in range(a.replicas) if r != a.unplanned)
            rec = s.unplanned_fault(a.unplanned)
            first = max(0, rec["fault_step"] - a.window // 4)
            s.await_(lambda: s.last_step(survivor) >= first + a.window, 1800, f"{a.window}-step window")
            rec["throughput"] = s.throughput_window(survivor, first, a.window)
        finally:
            s.finish()
        (s.dir / "unplanned_summary.json").write_text(json.dumps(rec, indent=1, default=str))
        print(json.dumps(rec, indent=1, default=str))
        return
    try:
        for i in range(a.faults):
            target = a.fault_step * (i + 1)
            s.await_(lambda: s.last_step(a.victim) >= target, 300, f"step {target}")
            if a.interval > 0:
                time.sleep(a.interval)
            rec = s.fault(a.victim, "worker" if a.worker_kill is not None else "launcher",
                          a.worker_kill or 0)
            results.append(rec)
            js = rec["joint_step"] + a.joint_commits
            s.await_(lambda: s.last_step(a.victim) >= js, 300, "joint commits")
        final = max(s.last_step(r) for r in range(a.replicas)) + 1
    finally:
        s.finish()
    print(json.dumps({"faults": results, "final_step": final}, indent=1))


if __name__ == "__main__":
    main()
