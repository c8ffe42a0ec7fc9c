"""Session evidence verifier (CPU only).

    python -m shift_b200.analysis.verify <session_dir> [--replicas 2] [--ranks 1]

Reads every JSONL file of a session and writes ``verify.json`` with
``checks{name: {pass, ...}}``.  The checks are those of the reference's
minimal verifier (shift_min/verify.py:162-345), restated for one box:

* all_ready             every rank of every replica reported ready in generation 0
* faults_injected       every injected fault is followed by a restart
* survivor_solo         survivors committed with fewer participants during a fault
* restored_hashes       every restored rank's state hashes equal the donor's snapshot
* rpo_zero              the restored step equals the survivor's last committed step:
                        no committed step is lost
* joint_hashes_equal    after recovery, commits at the same step carry equal model /
                        optimizer / scheduler hashes on every replica
* monotonic_steps       commit steps increase by one per rank and generation
* survivor_pid_stable   survivors kept their process ids across faults
* cleanup               supervisors ended with no children left
"""
from __future__ import annotations

import argparse
import json
from collections import defaultdict
from pathlib import Path

from ..control.event_reader import IncrementalReader


def verify(session_dir, replicas: int = 2, ranks: int = 1) -> dict:
    r = IncrementalReader(session_dir)
    r.poll()
    rows = r.all_rows
    checks = {}

    def add(name, ok, **info):
        checks[name] = dict(info, **{"pass": bool(ok)})

    ready0 = {(x["rid"], x["rank"]) for x in rows if x["kind"] == "ready" and x.get("generation") == 0}
    add("all_ready", len(ready0) == replicas * ranks, ready=sorted(ready0))
    injected = [x for x in rows if x["kind"] == "injected"]
    restarts = [x for x in rows if x["kind"] == "restart_requested"]
    add("faults_injected", len(restarts) >= len(injected), injected=len(injected), restarts=len(restarts))
    commits = [x for x in rows if x["kind"] == "commit"]
    restored = [x for x in rows if x["kind"] == "restored"]
    add("restored_hashes", all(x.get("hashes_match") for x in restored) and (not injected or restored),
        restored=len(restored), mismatches=[(x["rid"], x["rank"], x["step"]) for x in restored if not x.get("hashes_match")])
    # survivors committed solo while a peer was down
    solo_ok = True
    details = []
    for inj in injected:
        victim = inj["rid"]
        t0 = inj.get("fault_time", inj["time"])
        later = [c for c in commits if c["rid"] != victim and c["time"] > t0]
        solo = [c for c in later if c["participants"] < replicas]
        details.append({"victim": victim, "solo_commits": len(solo)})
        solo_ok &= bool(solo)
    add("survivor_solo", solo_ok, details=details)
    # RPO 0: restored step == last step committed by a survivor before the restore
    rpo = []
    for x in restored:
        before = [c["step"] for c in commits if c["rid"] != x["rid"] and c["time"] <= x["time"]]
        rpo.append({"rid": x["rid"], "rank": x["rank"], "restored_step": x["step"],
                    "survivor_last_commit": max(before) if before else 0})
    add("rpo_zero", all(e["restored_step"] == e["survivor_last_commit"] for e in rpo), details=rpo)
    # joint hashes after recovery
    by_step = defaultdict(dict)
    for c in commits:
        if c.get("hashes") and c["participants"] == replicas:
            by_step[(c["step"], c["rank"])][c["rid"]] = (c["hashes"].get("model"), c["hashes"].get("optimizer"),
                                                           c["hashes"].get("scheduler"))
    mism = []
    compared = 0
    for key, per in by_step.items():
        if len(per) == replicas:
            compared += 1
            if len(set(per.values())) != 1:
                mism.append(key)
    first_restore = min((x["time"] for x in restored), default=None)
    post = [k for k in by_step if first_restore is not None]
    add("joint_hashes_equal", not mism and compared > 0, compared_steps=compared, mismatched=mism[:10],
        post_recovery_steps=len(post))
    mono = True
    seq = defaultdict(list)
    for c in commits:
        seq[(c["rid"], c["rank"], c.get("generation"))].append(c["step"])
    breaks = []
    for k, s in seq.items():
        bad = [(a, b) for a, b in zip(s, s[1:]) if b != a + 1]
        if bad:
            mono = False
            breaks.append({"rid": k[0], "rank": k[1], "generation": k[2], "pairs": bad[:5]})
    add("monotonic_steps", mono, breaks=breaks)
    pids = defaultdict(set)
    for x in rows:
        if x["kind"] in ("commit", "ready") and "pid" in x:
            pids[(x["rid"], x["rank"], x.get("generation"))].add(x["pid"])
    add("survivor_pid_stable", all(len(v) == 1 for v in pids.values()))
    cleanup = [x for x in rows if x["kind"] == "cleanup"]
    add("cleanup", bool(cleanup) and all(not x.get("own_children") for x in cleanup), supervisors=len(cleanup))
    return {"checks": checks, "pass": all(c["pass"] for c in checks.values())}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("session_dir")
    ap.add_argument("--replicas", type=int, default=2)
    ap.add_argument("--ranks", type=int, default=1)
    a = ap.parse_args(argv)
    res = verify(a.session_dir, a.replicas, a.ranks)
    Path(a.session_dir, "verify.json").write_text(json.dumps(res, indent=1, sort_keys=True))
    print(json.dumps({k: v["pass"] for k, v in res["checks"].items()}, indent=1))
    return 0 if res["pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
