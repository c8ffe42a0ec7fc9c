"""Planned-handoff suites: every controlled scenario, repeated audited
handoffs, and alternating timing runs, each as its own planned session.

    python -m shift_b200.control.suite --phase scenarios|audit|timing [--root results/suite]
        [--post-steps N] [planned-session options: --model --device --nproc --gpus --module --train-args]

Phases (the reference's v2.1 suite, scripts/run_v21_suite.py:9-28, whose
outcomes RESULTS_V2_1.md:47-53 reports):

* ``scenarios`` -- P2 under each injected condition: the spare rejects its
  preparation, the spare misses its readiness deadline, the pre-copied state
  is stale, the gradient relay is rejected after the old epoch was revoked,
  and a slow compute step.  The first two must cancel the handoff and keep
  training in the old epoch; a stale state or a rejected relay must recover
  A+B in a new epoch with exact state; the slow step must still hand over.
* ``audit`` -- three healthy P2 handoffs, every commit hash-audited.
* ``timing`` -- P1f and P2 alternated (p1f p2 p2 p1f ...), the handoff
  interval of each, and the per-variant medians.

Each session's own summary decides its verdict (``pass``); the suite writes
``suite_<phase>.json`` with one row per session and ``all_pass``.
"""
from __future__ import annotations

import argparse
import json
import shlex
import statistics
import time
from pathlib import Path

from .planned import PlannedSession

SCENARIOS = ("relay-reject", "stale-state", "prepare-fail", "ready-timeout", "slow-compute")
TIMING_ORDER = ("p1f", "p2", "p2", "p1f", "p1f", "p2", "p2", "p1f", "p1f", "p2")


def jobs(phase: str) -> list[tuple[str, str]]:
    """(variant, scenario) of every session of a phase, in run order."""
    if phase == "scenarios":
        return [("p2", s) for s in SCENARIOS]
    if phase == "audit":
        return [("p2", "healthy")] * 3
    if phase == "timing":
        return [(v, "healthy") for v in TIMING_ORDER]
    raise ValueError(f"unknown phase {phase!r}")


def run_suite(phase: str, root, post_steps: int | None = None, make_session=PlannedSession, **session_kw) -> dict:
    root = Path(root)
    root.mkdir(parents=True, exist_ok=True)
    steps = post_steps if post_steps is not None else (50 if phase == "timing" else 10 if phase == "scenarios" else 6)
    rows = []
    for i, (variant, scenario) in enumerate(jobs(phase), 1):
        name = f"{phase}_{i:02d}_{variant}_{scenario.replace('-', '_')}"
        t0 = time.monotonic()
        try:
            s = make_session(root, name, variant, scenario, **session_kw)
            res = s.run(steps)
            row = {"name": name, "variant": variant, "scenario": scenario, "pass": bool(res.get("pass")),
                   "seconds": round(time.monotonic() - t0, 3),
                   "checks": {k: v["pass"] for k, v in res.get("checks", {}).items()}}
            for k in ("handoff_interval_s", "extra_interval_s", "cut", "cancelled", "final_step"):
                if k in res:
                    row[k] = res[k]
        except Exception as e:          # a session that crashed is a failed row, the suite goes on
            row = {"name": name, "variant": variant, "scenario": scenario, "pass": False,
                   "seconds": round(time.monotonic() - t0, 3), "error": repr(e)}
        rows.append(row)
    out = {"phase": phase, "post_steps": steps, "sessions": rows, "all_pass": all(r["pass"] for r in rows)}
    if phase == "timing":
        for v in ("p1f", "p2"):
            ivs = [r["handoff_interval_s"] for r in rows if r["variant"] == v and r.get("handoff_interval_s")]
            out[f"{v}_median_interval_s"] = statistics.median(ivs) if ivs else None
    (root / f"suite_{phase}.json").write_text(json.dumps(out, indent=1, default=str) + "\n")
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--phase", choices=["scenarios", "audit", "timing"], required=True)
    ap.add_argument("--root", default="results/suite")
    ap.add_argument("--post-steps", type=int, default=None)
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--nproc", type=int, default=1)
    ap.add_argument("--gpus", default="", help="A,B,C device lists, e.g. '0;1;2'")
    ap.add_argument("--module", default="shift_b200.ft.planned_train")
    ap.add_argument("--train-args", default="")
    a = ap.parse_args(argv)
    devices = {}
    if a.gpus:
        for role, lst in zip("ABC", a.gpus.split(";")):
            devices[role] = [int(x) for x in lst.split(",")]
    out = run_suite(a.phase, a.root, a.post_steps, model=a.model, device=a.device, nproc=a.nproc, devices=devices,
                    train_args=shlex.split(a.train_args), module=a.module)
    print(json.dumps(out, indent=1, default=str))
    return 0 if out["all_pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
