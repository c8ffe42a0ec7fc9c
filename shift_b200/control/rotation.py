"""v1 fail-stop rotation: seeded faults, cold / cpu / gpu standby restarts,
per-fault RPO and restore audits, and the disk-checkpoint restart scenario.

    python -m shift_b200.control.rotation --config cfg.json --session S \
        [--faults N] [--interval SEC | --fault-step K] [--backup-mode cold|cpu|gpu] [--seed 0] \
        [--checkpoint-restart]

Per fault (shift_full/rotation.py:129-239, rebuilt for one box):

1. the victim replica is drawn from ``random.Random(seed)``;
2. with ``--backup-mode cpu|gpu`` its next generation is prepared first as a
   standby (``PREPARE_g<G+1>``: the supervisor launches it with
   ``--standby``; a cpu standby waits before CUDA initialisation, a gpu one
   with its model built and warmed) and the controller waits until every
   rank reported ``standby_ready``;
3. the last joint commit (every rank of every replica, all replicas
   participating and contributing) is recorded, the victim's launcher tree
   is SIGKILLed (``KILL_g<G>``), the survivors must keep committing alone
   with unchanged PIDs;
4. ``RESTART_g<G+1>`` activates the standby (or cold-launches), every rank of
   the victim must report ``restored`` with matching state hashes at a step
   no earlier than the last joint commit before the fault (RPO 0), and the
   first joint commit after the restored step closes the fault.

Results go to ``fault_results.json``: fault -> solo / ready / restored /
joint times, request -> loaded, the restored step against the committed
step, and the standby preparation time.  ``--checkpoint-restart`` runs the
disk baseline instead: both replicas are killed after their trainers wrote
and re-read a checkpoint (``--checkpoint-step``), restart from it
(``--resume-checkpoint``) and must commit jointly again
(shift_full/control.py:340-355).
"""
from __future__ import annotations

import argparse
import json
import random
import statistics
import time

from .session import Session, joint_boundary


class Rotation:
    def __init__(self, session: Session, backup_mode: str = "cold", seed: int = 0, solo_timeout: float = 120.0,
                 step_timeout: float = 300.0):
        if backup_mode not in ("cold", "cpu", "gpu"):
            raise ValueError(f"backup mode must be cold, cpu or gpu, got {backup_mode!r}")
        self.s = session
        self.mode = backup_mode
        self.rng = random.Random(seed)
        self.solo_timeout = solo_timeout
        self.step_timeout = step_timeout
        self.results: list[dict] = []

    # ------------------------------------------------------------------ evidence helpers
    def _rank_rows(self, kind, rid, gen):
        return [r for r in self.s.reader.rows(kind, rid=rid, generation=gen)]

    def last_joint_step(self, before_time: float | None = None) -> int:
        """Largest step every rank of every replica (current generations)
        committed with all replicas participating and contributing."""
        s = self.s
        per = []
        for rid in range(s.replicas):
            gen = s.generation[rid]
            rows = [c for rank in range(s.ranks()) for c in s.commits(rid, gen, rank=rank)
                    if before_time is None or c.get("time", 0) <= before_time]
            steps = {}
            for c in rows:
                if c.get("participants") == s.replicas and c.get("contributed") is not False:
                    steps.setdefault(c["step"], set()).add(c.get("rank", 0))
            per.append({st for st, rk in steps.items() if len(rk) == s.ranks()})
        common = set.intersection(*per) if per else set()
        return max(common) if common else 0

    def _ready_pids(self, rid):
        gen = self.s.generation[rid]
        return {r["rank"]: r["pid"] for r in self._rank_rows("ready", rid, gen)}

    # ------------------------------------------------------------------ one fault
    def fault(self, index: int) -> dict:
        s = self.s
        R, ranks = s.replicas, s.ranks()
        target = self.rng.randrange(R)
        healthy = [r for r in range(R) if r != target]
        gen = s.generation[target]
        s.log("fault_planned", index=index, target=target, generation=gen, backup_mode=self.mode)
        t_prep = time.time()
        standby_rows = []
        if self.mode != "cold":
            s.marker(f"PREPARE_g{gen + 1}_r{target}", self.mode)
            s.await_(lambda: len({e["rank"] for e in self._rank_rows("standby_ready", target, gen + 1)}) == ranks,
                     self.step_timeout, f"fault {index}: {self.mode} standby ready")
            standby_rows = self._rank_rows("standby_ready", target, gen + 1)
        prep_s = time.time() - t_prep
        s.await_(lambda: self.last_joint_step() > 0, self.step_timeout, f"fault {index}: a joint commit")
        committed = self.last_joint_step()
        healthy_pids = {r: self._ready_pids(r) for r in healthy}
        s.marker(f"KILL_g{gen}_r{target}")
        s.await_(lambda: self.s.reader.rows("injected", rid=target, generation=gen), 60, f"fault {index}: injection")
        fault_at = s.reader.rows("injected", rid=target, generation=gen)[0]["fault_time"]
        committed = max(committed, self.last_joint_step(before_time=fault_at))
        # the survivors keep training alone
        s.await_(lambda: all(any(c["participants"] == R - 1 and c["step"] > committed
                                 for c in s.commits(h, s.generation[h])) for h in healthy),
                 self.solo_timeout, f"fault {index}: solo commits")
        solo_at = min(min(c["time"] for c in s.commits(h, s.generation[h])
                          if c["participants"] == R - 1 and c["step"] > committed) for h in healthy)
        request_at = time.time()
        s.marker(f"RESTART_g{gen + 1}_r{target}")
        s.generation[target] = gen + 1
        s.await_(lambda: len({e["rank"] for e in self._rank_rows("ready", target, gen + 1)}) == ranks,
                 self.step_timeout, f"fault {index}: replacement ready")
        s.await_(lambda: len({e["rank"] for e in self._rank_rows("restored", target, gen + 1)}) == ranks,
                 self.step_timeout, f"fault {index}: restored")
        restores = self._rank_rows("restored", target, gen + 1)
        loaded = self._rank_rows("state_loaded", target, gen + 1)
        requests = self._rank_rows("recovery_request", target, gen + 1)
        ready = self._rank_rows("ready", target, gen + 1)
        restored_steps = {e["step"] for e in restores}
        audit_ok = all(e.get("hashes_match") for e in restores)
        rpo_ok = len(restored_steps) == 1 and min(restored_steps) >= committed
        rstep = max(restored_steps)
        s.await_(lambda: s._joint(target, gen + 1, rstep) is not None, self.step_timeout, f"fault {index}: joint")
        jstep, jtime = s._joint(target, gen + 1, rstep)
        pids_same = all(c.get("pid") == healthy_pids[h].get(c.get("rank", 0))
                        for h in healthy for rank in range(ranks) for c in s.commits(h, s.generation[h], rank=rank))
        res = dict(index=index, target=target, backup_mode=self.mode, generation=gen + 1,
                   committed_before_fault=committed, restored_step=rstep, first_joint_step=jstep,
                   rpo_steps=max(0, committed - min(restored_steps)), rpo_zero=rpo_ok, restore_hashes_match=audit_ok,
                   healthy_pids_unchanged=pids_same, preparation_seconds=prep_s,
                   standby_resources=[{k: e.get(k) for k in ("rank", "mode", "cpu_maxrss_kib", "cuda_allocated_bytes")}
                                      for e in standby_rows],
                   fault_time=fault_at, solo_time=solo_at, request_time=request_at,
                   ready_time=max(e["time"] for e in ready), loaded_time=max(e["time"] for e in restores),
                   state_loaded_time=max(e["time"] for e in loaded) if loaded else None,
                   recovery_request_time=min(e["time"] for e in requests) if requests else None, joint_time=jtime)
        res["fault_to_solo_seconds"] = solo_at - fault_at
        res["fault_to_joint_seconds"] = jtime - fault_at
        res["request_to_ready_seconds"] = res["ready_time"] - request_at
        res["request_to_loaded_seconds"] = res["loaded_time"] - request_at
        if res["recovery_request_time"] is not None and res["state_loaded_time"] is not None:
            res["recovery_request_to_loaded_seconds"] = res["state_loaded_time"] - res["recovery_request_time"]
        res["pass"] = bool(rpo_ok and audit_ok and pids_same)
        self.results.append(res)
        (s.dir / "fault_results.json").write_text(json.dumps(self.results, indent=1, default=str) + "\n")
        s.log("rotation_verified", **{k: v for k, v in res.items() if k != "standby_resources"})
        return res

    # ------------------------------------------------------------------ disk checkpoint baseline
    def checkpoint_restart(self, timeout: float = 600.0) -> dict:
        """Both replicas' trainers saved (and re-read) a disk checkpoint at
        ``--checkpoint-step``; two steps later both are killed and restarted
        from it, and must train jointly again."""
        s = self.s
        R, ranks = s.replicas, s.ranks()
        s.await_(lambda: all(len({e["rank"] for e in self._rank_rows("checkpoint_loaded", r, 0)}) == ranks
                             for r in range(R)), timeout, "checkpoint written and re-read")
        ck = min(e["step"] for r in range(R) for e in self._rank_rows("checkpoint_loaded", r, 0))
        s.await_(lambda: self.last_joint_step() >= ck + 2, timeout, "two commits past the checkpoint")
        for r in range(R):
            s.marker(f"EXPECT_PEER_FAILURE_g0_r{r}")
        t_kill = time.time()
        for r in range(R):
            s.marker(f"KILL_g0_r{r}")
        s.await_(lambda: all(s.reader.rows("injected", rid=r, generation=0) for r in range(R)), 60, "both killed")
        for r in range(R):
            s.marker(f"RESTART_g1_r{r}", "resume_checkpoint")
            s.generation[r] = 1
        s.await_(lambda: all(len({e["rank"] for e in self._rank_rows("checkpoint_resumed", r, 1)}) == ranks
                             for r in range(R)), timeout, "resumed from the checkpoint")
        resumed = [e for r in range(R) for e in self._rank_rows("checkpoint_resumed", r, 1)]

        def joint_now():
            rows = [c for r in range(R) for rank in range(ranks) for c in s.commits(r, 1, rank=rank)]
            return joint_boundary(rows, 0, 1, ck, R, ranks)

        # the replicas come back at their own pace: one may commit alone (and
        # the other heal from it) before the first commit they make together
        s.await_(lambda: joint_now() is not None, timeout, "first joint commit after resume")
        joint = joint_now()
        res = {"checkpoint_step": ck, "resumed_steps": sorted({e["step"] for e in resumed}),
               "resume_seconds": statistics.median(e["seconds"] for e in resumed),
               "kill_to_first_joint_seconds": (joint[1] - t_kill) if joint else None,
               "first_joint_step": joint[0] if joint else None,
               "pass": bool(joint) and all(e["step"] == ck for e in resumed)}
        (s.dir / "checkpoint_restart.json").write_text(json.dumps(res, indent=1) + "\n")
        s.log("checkpoint_restart_verified", **res)
        return res


def summarize(results: list[dict]) -> dict:
    """p50 / p95 of fault -> first joint commit and the audit tallies."""
    xs = sorted(r["fault_to_joint_seconds"] for r in results)

    def pct(q):
        return xs[min(len(xs) - 1, int(round(q * (len(xs) - 1))))] if xs else None

    return {"faults": len(results), "fault_to_joint_p50": statistics.median(xs) if xs else None,
            "fault_to_joint_p95": pct(0.95), "rpo_zero": sum(r["rpo_zero"] for r in results),
            "restore_audits_pass": sum(r["restore_hashes_match"] for r in results),
            "all_pass": all(r["pass"] for r in results),
            "backup_modes": sorted({r["backup_mode"] for r in results})}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", required=True)
    ap.add_argument("--session", required=True)
    ap.add_argument("--root", default="results")
    ap.add_argument("--replicas", type=int, default=2)
    ap.add_argument("--faults", type=int, default=3)
    ap.add_argument("--interval", type=float, default=0.0, help="seconds between faults (after a recovery)")
    ap.add_argument("--fault-step", type=int, default=3, help="joint commits between faults")
    ap.add_argument("--backup-mode", choices=("cold", "cpu", "gpu"), default="cold")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--checkpoint-restart", action="store_true")
    ap.add_argument("--seconds", type=float, default=1800)
    a = ap.parse_args(argv)
    s = Session(a.root, a.session, a.config, a.replicas, seconds=a.seconds)
    rot = Rotation(s, a.backup_mode, a.seed)
    s.start()
    out = {}
    try:
        if a.checkpoint_restart:
            out["checkpoint_restart"] = rot.checkpoint_restart()
        else:
            for i in range(a.faults):
                base = rot.last_joint_step()
                s.await_(lambda: rot.last_joint_step() >= base + a.fault_step, 600, f"{a.fault_step} joint commits")
                if a.interval > 0:
                    time.sleep(a.interval)
                rot.fault(i)
            out["summary"] = summarize(rot.results)
            out["faults"] = rot.results
    finally:
        s.finish()
    (s.dir / "rotation_summary.json").write_text(json.dumps(out, indent=1, default=str) + "\n")
    print(json.dumps(out.get("summary", out), indent=1, default=str))


if __name__ == "__main__":
    main()
