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


def _leaves(tree, prefix="", keep_scalars: bool = False):
    """(path, leaf) pairs in a fixed order.  Tensors always; with
    ``keep_scalars`` also every non-container leaf (ints, floats, strings)."""
    if isinstance(tree, torch.Tensor):
        yield prefix, tree
    elif isinstance(tree, dict):
        for k in sorted(tree, key=lambda x: (type(x).__name__, str(x))):
            yield from _leaves(tree[k], f"{prefix}/{k}", keep_scalars)
    elif isinstance(tree, (list, tuple)):
        for i, v in enumerate(tree):
            yield from _leaves(v, f"{prefix}/{i}", keep_scalars)
    elif keep_scalars:
        yield prefix, tree


def _bitwise_equal(x, y) -> tuple[bool, str]:
    """Strict equality of two leaves: same type; tensors of the same dtype,
    shape and layout with identical bytes (so -0.0 differs from 0.0 and NaNs
    compare by payload); other leaves by ``==``."""
    if isinstance(x, torch.Tensor) != isinstance(y, torch.Tensor):
        return False, "tensor vs non-tensor"
    if not isinstance(x, torch.Tensor):
        return (type(x) is type(y) and x == y), f"{x!r} != {y!r}"
    if x.dtype != y.dtype:
        return False, f"dtype {x.dtype} vs {y.dtype}"
    if x.shape != y.shape or x.layout != y.layout:
        return False, f"shape/layout {tuple(x.shape)}/{x.layout} vs {tuple(y.shape)}/{y.layout}"
    xa, ya = x.detach().cpu().contiguous(), y.detach().cpu().contiguous()
    if xa.numel() == 0:
        return True, ""
    same = torch.equal(xa.flatten().view(torch.uint8), ya.flatten().view(torch.uint8))
    return same, "" if same else "bytes differ"


def compare_strict(a, b) -> dict:
    """Bitwise comparison of two trees, non-tensor leaves included."""
    la, lb = dict(_leaves(a, keep_scalars=True)), dict(_leaves(b, keep_scalars=True))
    if la.keys() != lb.keys():
        return {"pass": False, "error": "different structure", "only_a": sorted(la.keys() - lb.keys())[:5],
                "only_b": sorted(lb.keys() - la.keys())[:5]}
    diffs = []
    for k in la:
        ok, why = _bitwise_equal(la[k], lb[k])
        if not ok:
            diffs.append({"leaf": k, "why": why})
    return {"pass": not diffs, "differing_leaves": len(diffs), "first": diffs[:5], "leaves": len(la)}


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
    """``strict``: bitwise equality of every leaf -- dtypes, shapes and
    bytes of tensors, and non-tensor leaves by ``==`` (the reference's strict
    fp32 comparison, shift_full/compare_reference.py:160-190), which a flat
    run and a cross-replica average are expected to fail from the first
    update whose reductions round in a different order."""
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
            if strict:
                res = {f: compare_strict(a[f], b[f]) for f in TOLERANCES}
            else:
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
    ap.add_argument("--strict", action="store_true", help="bitwise equality of every leaf (dtype, shape, bytes; non-tensor leaves by ==)")
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
