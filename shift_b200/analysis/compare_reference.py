"""Numerical oracle: compare two runs' per-step reference dumps.

    python -m shift_b200.analysis.compare_reference RUN_A RUN_B [--steps 1,2,3] [--ranks 1] [--out report.json]

Each run directory holds ``reference_step<k>_r<rank>.pt`` written by the
trainer's ``--reference-dump`` (the averaged gradient and the committed model,
optimizer and scheduler state after step k).  Typical use: the flat baseline
(``--mode flat``: one process, the whole global batch, no Manager) against
the fault-tolerant run (two replicas through the quorum and the cross-replica
average).  Tolerances follow the reference's comparison
(shift_full/compare_reference.py:17-24): gradients atol 1e-5 / rtol 1e-3,
model 1e-6 / 1e-4, optimizer 1e-5 / 1e-3, scheduler exact.
"""
from __future__ import annotations

import argparse
import json
from pathlib import Path

import torch

TOLERANCES = {"gradients": (1e-5, 1e-3), "model": (1e-6, 1e-4), "optimizer": (1e-5, 1e-3)}


def _leaves(tree, prefix=""):
    if isinstance(tree, torch.Tensor):
        yield prefix, tree
    elif isinstance(tree, dict):
        for k in sorted(tree, key=lambda x: (type(x).__name__, str(x))):
            yield from _leaves(tree[k], f"{prefix}/{k}")
    elif isinstance(tree, (list, tuple)):
        for i, v in enumerate(tree):
            yield from _leaves(v, f"{prefix}/{i}")


def compare_tensors(a, b, atol: float, rtol: float) -> dict:
    """Worst element over all leaves: |a - b| <= atol + rtol * |b|."""
    la, lb = dict(_leaves(a)), dict(_leaves(b))
    if la.keys() != lb.keys():
        return {"pass": False, "error": "different structure", "only_a": sorted(la.keys() - lb.keys())[:5],
                "only_b": sorted(lb.keys() - la.keys())[:5]}
    worst, worst_key, ok = 0.0, None, True
    for k in la:
        x, y = la[k].float(), lb[k].float()
        if x.shape != y.shape:
            return {"pass": False, "error": f"shape mismatch at {k}"}
        if x.numel() == 0:
            continue
        excess = ((x - y).abs() - (atol + rtol * y.abs())).max().item()
        if excess > worst or worst_key is None:
            worst, worst_key = excess, k
        ok &= excess <= 0.0
    return {"pass": bool(ok), "worst_excess": worst, "worst_leaf": worst_key, "leaves": len(la)}


def compare_runs(run_a, run_b, steps=None, ranks: int = 1, strict: bool = False) -> dict:
    """``strict``: zero tolerances (bitwise equality of every leaf) -- the
    reference's strict-fp32 comparison, which a flat run and a cross-replica
    average are expected to fail from the first update whose reductions
    round in a different order."""
    run_a, run_b = Path(run_a), Path(run_b)
    tol = {f: (0.0, 0.0) for f in TOLERANCES} if strict else TOLERANCES
    if steps is None:
        steps = sorted(int(p.name.split("_step")[1].split("_")[0]) for p in run_a.glob("reference_step*_r0.pt"))
    out = {"steps": {}, "tolerances": tol, "strict": strict}
    all_ok = bool(steps)
    for k in steps:
        for r in range(ranks):
            pa, pb = run_a / f"reference_step{k}_r{r}.pt", run_b / f"reference_step{k}_r{r}.pt"
            if not pa.exists() or not pb.exists():
                out["steps"][f"{k}/{r}"] = {"pass": False, "error": "missing dump"}
                all_ok = False
                continue
            a = torch.load(pa, weights_only=False)
            b = torch.load(pb, weights_only=False)
            res = {f: compare_tensors(a[f], b[f], *tol[f]) for f in TOLERANCES}
            res["scheduler"] = {"pass": a["scheduler"] == b["scheduler"]}
            res["pass"] = all(v["pass"] for v in res.values() if isinstance(v, dict))
            out["steps"][f"{k}/{r}"] = res
            all_ok &= res["pass"]
    out["pass"] = all_ok
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("run_a")
    ap.add_argument("run_b")
    ap.add_argument("--steps", default="")
    ap.add_argument("--ranks", type=int, default=1)
    ap.add_argument("--strict", action="store_true", help="zero tolerances (bitwise equality)")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    steps = [int(x) for x in a.steps.split(",") if x] or None
    res = compare_runs(a.run_a, a.run_b, steps, a.ranks, a.strict)
    text = json.dumps(res, indent=1, default=str)
    if a.out:
        Path(a.out).write_text(text)
    print(text)
    return 0 if res["pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
