"""Trajectory summary: did the flat baseline and the fault-tolerant run train
on the same thing?

    python -m shift_b200.analysis.trajectory FLAT_DIR SHIFT_DIR [--comparison report.json] [--out summary.json]

The numerical oracle (``compare_reference``) checks that the two runs end each
step with the same gradients and state within tolerance.  This summary checks
the inputs of that comparison from the runs' event logs
(``events_g<G>_r<R>.jsonl``), the role of the reference's
shift_full/summarize_trajectory.py:300-358:

* ``input_read``: both runs have event logs and every line parses;
* ``same_initial_state``: the generation-0 ``ready`` digests of model,
  optimizer, scheduler and progress (trainer ``--audit-state``) are equal in
  the flat run and in every replica of the fault-tolerant run;
* ``step_coverage``: both runs planned the same pre-update steps;
* ``same_batch_plans``: per step, the flat run's sample ids equal the union
  of the replicas' sample ids, and no sample is trained twice in a step;
* ``same_routing``: per (step, sample, MoE layer), the digest of the router's
  top-k expert indices is the same in both runs (trainer ``--trace-routing``);
* ``participants_and_global_batch``: every committed step of the
  fault-tolerant run had all replicas participating and covered the flat
  run's global batch;
* ``numerical_comparison``: the ``compare_reference`` report passes (read
  from ``--comparison``, or computed from the runs' reference dumps).

A step that was attempted more than once (a skipped commit) counts with its
last attempt.  fp32 reduction order differs between the runs (one process
against a cross-replica average), so agreement of plans and routing does not
imply bitwise-equal state; that is what the tolerances of the numerical
comparison are for.
"""
from __future__ import annotations

import argparse
import json
from collections import defaultdict
from pathlib import Path

STATE_FIELDS = ("model", "optimizer", "scheduler", "progress")


def read_events(directory) -> tuple[list[dict], list[str], int]:
    """All event rows under ``directory`` (recursively), parse errors, file count."""
    rows, errors = [], []
    files = sorted(Path(directory).rglob("events_g*_r*.jsonl"))
    for path in files:
        try:
            with open(path, encoding="utf-8") as f:
                for n, line in enumerate(f, 1):
                    if not line.strip():
                        continue
                    try:
                        v = json.loads(line)
                    except ValueError as exc:
                        errors.append(f"{path}:{n}: {type(exc).__name__}")
                        continue
                    if isinstance(v, dict):
                        rows.append(v)
        except OSError as exc:
            errors.append(f"{path}: {exc}")
    return rows, errors, len(files)


def _gen0(rows, kind):
    return [r for r in rows if r.get("kind") == kind and int(r.get("generation", 0) or 0) == 0]


def _initial_state(flat_rows, shift_rows) -> dict:
    flat = [r for r in _gen0(flat_rows, "ready") if r.get("hashes")]
    shift = [r for r in _gen0(shift_rows, "ready") if r.get("hashes")]
    if not flat or not shift:
        return {"pass": False, "error": "ready rows without state digests (run both with --audit-state)",
                "flat_rows": len(flat), "shift_rows": len(shift)}
    ref = flat[0]["hashes"]
    fields = [f for f in STATE_FIELDS if f in ref]
    unequal = []
    for r in shift:
        for f in fields:
            if r["hashes"].get(f) != ref.get(f):
                unequal.append({"rid": r.get("rid"), "rank": r.get("rank"), "field": f})
    return {"pass": bool(fields) and not unequal, "fields": fields, "replica_rows": len(shift),
            "unequal": unequal[:20]}


def _plans(rows) -> dict:
    """step -> {rid: sample ids of the last attempt}."""
    out: dict = defaultdict(dict)
    for r in _gen0(rows, "batch_plan"):
        out[int(r["step"])][r.get("rid", 0)] = list(r.get("sample_ids") or [])
    return out


def _batch_plans(flat_rows, shift_rows) -> tuple[dict, dict, list[int]]:
    fp, sp = _plans(flat_rows), _plans(shift_rows)
    steps = sorted(set(fp) & set(sp))
    coverage = {"pass": bool(steps) and set(fp) == set(sp), "flat_steps": sorted(fp), "shift_steps": sorted(sp)}
    unequal, duplicated = [], []
    for s in steps:
        flat_ids = sorted(i for ids in fp[s].values() for i in ids)
        shift_ids = [i for ids in sp[s].values() for i in ids]
        if len(set(shift_ids)) != len(shift_ids):
            duplicated.append(s)
        if flat_ids != sorted(shift_ids):
            unequal.append({"step": s, "flat": flat_ids, "shift": sorted(shift_ids)})
    plans = {"pass": bool(steps) and not unequal and not duplicated, "steps": len(steps),
             "unequal": unequal[:10], "duplicated_steps": duplicated}
    return coverage, plans, steps


def _routing_map(rows) -> dict:
    out = {}
    for r in _gen0(rows, "routing"):
        out[(int(r["step"]), int(r["sample"]), str(r["layer"]))] = r.get("topk_hash")
    return out


def _routing(flat_rows, shift_rows, steps) -> dict:
    fm, sm = _routing_map(flat_rows), _routing_map(shift_rows)
    if not fm or not sm:
        return {"pass": False, "error": "no routing events (run both with --trace-routing)",
                "flat_keys": len(fm), "shift_keys": len(sm)}
    keep = set(steps)
    fk = {k for k in fm if k[0] in keep}
    sk = {k for k in sm if k[0] in keep}
    unequal = sorted(k for k in fk & sk if fm[k] != sm[k])
    return {"pass": bool(fk) and fk == sk and not unequal, "keys": len(fk & sk),
            "flat_only": [list(k) for k in sorted(fk - sk)[:10]], "shift_only": [list(k) for k in sorted(sk - fk)[:10]],
            "unequal": [list(k) for k in unequal[:10]]}


def _participants(flat_rows, shift_rows, steps) -> dict:
    replicas = {r.get("rid") for r in _gen0(shift_rows, "ready")}
    commits = _gen0(shift_rows, "commit")
    bad = []
    per_step = defaultdict(set)
    for r in commits:
        per_step[int(r["step"])].add(r.get("rid"))
        if r.get("participants") != len(replicas):
            bad.append({"step": r["step"], "rid": r.get("rid"), "participants": r.get("participants")})
    fp, sp = _plans(flat_rows), _plans(shift_rows)
    short = [s for s in steps
             if sum(len(v) for v in sp[s].values()) != sum(len(v) for v in fp[s].values())]
    # commit rows carry the post-update step: step s+1 commits plan s
    missing = [s for s in steps if per_step.get(s + 1, set()) != replicas]
    return {"pass": bool(commits) and not bad and not short and not missing, "replicas": len(replicas),
            "commits": len(commits), "wrong_participants": bad[:10], "short_global_batch_steps": short,
            "steps_without_every_replica": missing}


def _numerical(flat_dir, shift_dir, comparison) -> dict:
    if comparison is None:
        if not list(Path(flat_dir).glob("reference_step*_r0.pt")):
            return {"pass": False, "error": "no comparison report and no reference dumps (--reference-dump)"}
        from .compare_reference import compare_runs
        comparison = compare_runs(flat_dir, shift_dir)
    elif not isinstance(comparison, dict):
        try:
            comparison = json.loads(Path(comparison).read_text())
        except (OSError, ValueError) as exc:
            return {"pass": False, "error": f"{type(exc).__name__}: {exc}"}
    return {"pass": comparison.get("pass") is True, "steps": sorted(comparison.get("steps", {}))}


def summarize(flat_dir, shift_dir, comparison=None) -> dict:
    flat_rows, ferr, fn = read_events(flat_dir)
    shift_rows, serr, sn = read_events(shift_dir)
    coverage, plans, steps = _batch_plans(flat_rows, shift_rows)
    checks = {
        "input_read": {"pass": fn > 0 and sn > 0 and not ferr and not serr, "flat_files": fn, "shift_files": sn,
                       "errors": (ferr + serr)[:10]},
        "same_initial_state": _initial_state(flat_rows, shift_rows),
        "step_coverage": coverage,
        "same_batch_plans": plans,
        "same_routing": _routing(flat_rows, shift_rows, steps),
        "participants_and_global_batch": _participants(flat_rows, shift_rows, steps),
        "numerical_comparison": _numerical(flat_dir, shift_dir, comparison),
    }
    return {"pass": all(c["pass"] for c in checks.values()), "checks": checks,
            "note": "fp32 reduction order differs between the runs; plans and routing agreeing does not imply "
                    "bitwise-equal state (the numerical comparison has tolerances)"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("flat_dir")
    ap.add_argument("shift_dir")
    ap.add_argument("--comparison", default=None, help="compare_reference report JSON")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    rep = summarize(a.flat_dir, a.shift_dir, a.comparison)
    text = json.dumps(rep, indent=1, default=str)
    if a.out:
        Path(a.out).write_text(text)
    print(json.dumps({"pass": rep["pass"], "checks": {k: v["pass"] for k, v in rep["checks"].items()}}))
    return 0 if rep["pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
