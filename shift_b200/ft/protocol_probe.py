"""Protocol negatives of the planned handoff's epoch fence.

    python -m shift_b200.ft.protocol_probe [--out negatives.json]

Runs every request the ``EpochGate`` must refuse -- the list of the
reference's scripts/probe_planned_protocol.py:5-16 (stale or skipped epoch,
stale state, unready C, old B, old A, cancel after activation) plus a
repeated activation and a C that acts before it owns the epoch -- and the
two transitions it must allow, each on a fresh gate.  The JSON report has one
``checks`` entry per case; the exit code is 0 when all pass.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

from .handoff import EpochGate


def _activated() -> EpochGate:
    g = EpochGate()
    g.activate(1, 5, 5, True)
    return g


# (name, action on a gate, gate factory): each action must raise ValueError
NEGATIVES = [
    ("skipped_epoch", lambda g: g.activate(2, 5, 5, True), EpochGate),
    ("stale_epoch", lambda g: g.activate(0, 5, 5, True), EpochGate),
    ("stale_state", lambda g: g.activate(1, 5, 4, True), EpochGate),
    ("unready_c", lambda g: g.activate(1, 5, 5, False), EpochGate),
    ("c_before_activation", lambda g: g.authorize("C", 0), EpochGate),
    ("old_b_after_activation", lambda g: g.authorize("B", 1), _activated),
    ("old_a_epoch", lambda g: g.authorize("A", 0), _activated),
    ("repeated_activation", lambda g: g.activate(1, 5, 5, True), _activated),
    ("cancel_after_activation", lambda g: g.cancel(), _activated),
]


def run() -> dict:
    checks = {}
    for name, action, make in NEGATIVES:
        g = make()
        before = (g.epoch, g.members)
        try:
            action(g)
            checks[name] = {"pass": False, "error": "accepted"}
        except ValueError as exc:
            # a refusal leaves the gate as it was
            checks[name] = {"pass": (g.epoch, g.members) == before, "refused": str(exc)}
    g = EpochGate()
    checks["cancel_before_activation"] = {"pass": g.cancel() == ("A", "B") and g.epoch == 0}
    g = _activated()
    try:
        g.authorize("A", 1)
        g.authorize("C", 1)
        ok = g.members == ("A", "C") and g.epoch == 1 and g.step == 5
    except ValueError:
        ok = False
    checks["activation_hands_b_to_c"] = {"pass": ok}
    return {"pass": all(c["pass"] for c in checks.values()), "negatives": len(NEGATIVES), "checks": checks}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    rep = run()
    text = json.dumps(rep, indent=1)
    if a.out:
        Path(a.out).write_text(text)
    print(json.dumps({"pass": rep["pass"], "negatives": rep["negatives"]}))
    return 0 if rep["pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
