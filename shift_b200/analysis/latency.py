"""Recovery and step latencies of a fault-tolerance session.

    python -m shift_b200.analysis.latency SESSION_DIR [--out latency.json]

From the controller's ``fault_recovered`` records: fault -> solo commit,
fault -> restored (state loaded and audited on every rank) and fault -> first
joint commit, with median / p95 over the session's faults; from each
replica's rank-0 commits: the steady commit interval (median / p95) outside
the fault windows.  Mirrors the reference's latency report
(shift_full/latency.py) for an in-box session.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

from ..control.event_reader import IncrementalReader


def _pct(xs, q):
    if not xs:
        return None
    xs = sorted(xs)
    i = min(len(xs) - 1, max(0, int(round(q * (len(xs) - 1)))))
    return xs[i]


def summarize(session_dir) -> dict:
    r = IncrementalReader(session_dir)
    r.poll()
    rows = r.all_rows
    faults = [x for x in rows if x["kind"] == "fault_recovered"]
    out = {"faults": len(faults)}
    for name, a, b in (("fault_to_solo_s", "fault_time", "solo_time"),
                       ("fault_to_restored_s", "fault_time", "restored_time"),
                       ("fault_to_joint_s", "fault_time", "joint_time")):
        xs = [f[b] - f[a] for f in faults if a in f and b in f]
        out[name] = {"median": _pct(xs, 0.5), "p95": _pct(xs, 0.95), "max": max(xs) if xs else None}
    windows = [(f["fault_time"], f["joint_time"]) for f in faults if "fault_time" in f and "joint_time" in f]
    per_replica = {}
    for rid in sorted({x.get("rid") for x in rows if x["kind"] == "commit" and x.get("rid") is not None}):
        c = sorted((x for x in rows if x["kind"] == "commit" and x.get("rid") == rid and x.get("rank") == 0),
                   key=lambda x: x["time"])
        gaps = [b["time"] - a["time"] for a, b in zip(c, c[1:])
                if not any(s - 1.0 <= b["time"] <= e + 1.0 for s, e in windows)]
        per_replica[str(rid)] = {"commits": len(c), "interval_median_s": _pct(gaps, 0.5),
                                 "interval_p95_s": _pct(gaps, 0.95)}
    out["commit_intervals"] = per_replica
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("session_dir")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    res = summarize(a.session_dir)
    text = json.dumps(res, indent=1)
    if a.out:
        Path(a.out).write_text(text)
    print(text)


if __name__ == "__main__":
    main()
