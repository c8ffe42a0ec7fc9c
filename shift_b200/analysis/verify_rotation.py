"""Verification of a continuous-rotation (multi-cycle planned handoff) session.

    python -m shift_b200.analysis.verify_rotation SESSION_DIR [--variant p2] [--max-gap-factor 20]

Checks, per round and over the whole run (cf. shift_full/verify_rotation.py):
* every round's receiver restored the donor's state hashes and then committed
  bit-exactly with A at the same steps (``round<r>_state_exact``)
* A's commit steps increase by one across every cut (no step lost or repeated)
* no gap between consecutive A commits exceeds ``max_gap_factor`` x the
  median steady interval (the handoff window included)
* hash completeness: every commit of A and of every receiver carries model /
  optimizer / scheduler hashes (audited runs)
* every retired donor logged its retirement and no retired process committed
  after its round's cut
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

from ..control.event_reader import IncrementalReader
from ..control.planned import summarize_cycles


def verify(session_dir, variant: str = "p2", max_gap_factor: float = 20.0, nproc: int = 1) -> dict:
    r = IncrementalReader(session_dir)
    r.poll()
    rows = r.all_rows
    cuts = sorted({x["step"] for x in rows if x["kind"] == "planned_cut_selected" and x.get("rid") == 0})
    res = summarize_cycles(r, variant, {"cuts": cuts}, nproc)
    checks = res["checks"]
    a0 = sorted((x for x in rows if x["kind"] == "commit" and x["rid"] == 0 and x["rank"] == 0),
                key=lambda x: x["time"])
    gaps = [b["time"] - a["time"] for a, b in zip(a0, a0[1:])]
    med = sorted(gaps)[len(gaps) // 2] if gaps else 0.0
    checks["bounded_gaps"] = {"pass": bool(gaps) and max(gaps) <= max_gap_factor * max(med, 1e-3),
                              "max_gap_s": max(gaps) if gaps else None, "median_s": med}
    audited = [x for x in rows if x["kind"] == "commit" and x.get("hashes") is not None]
    complete = all(all(k in x["hashes"] for k in ("model", "optimizer", "scheduler")) for x in audited
                   if x["hashes"])
    checks["hash_completeness"] = {"pass": complete and any(x["hashes"] for x in audited)}
    retired = [x for x in rows if x["kind"] == "stopped" and x.get("retired")]
    late = []
    for x in retired:
        gen = x["generation"]
        late += [c for c in rows if c["kind"] == "commit" and c["generation"] == gen and c["rid"] == x["rid"]
                 and c["time"] > x["time"]]
    checks["retired_no_late_commits"] = {"pass": not late and len(retired) >= len(cuts) * nproc,
                                        "retired": len(retired)}
    res["pass"] = all(c["pass"] for c in checks.values())
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("session_dir")
    ap.add_argument("--variant", default="p2")
    ap.add_argument("--max-gap-factor", type=float, default=20.0)
    ap.add_argument("--nproc", type=int, default=1)
    a = ap.parse_args(argv)
    res = verify(a.session_dir, a.variant, a.max_gap_factor, a.nproc)
    (Path(a.session_dir) / "verify_rotation.json").write_text(json.dumps(res, indent=1, default=str))
    print(json.dumps({k: v["pass"] for k, v in res["checks"].items()}, indent=1))
    return 0 if res["pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
