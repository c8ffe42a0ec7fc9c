"""Trace one AdamW coordinate through a step in two runs' reference dumps.

    python -m shift_b200.analysis.adam_trace FLAT_DIR SHIFT_DIR --step 3 [--rank 0] [--param NAME --index I]

When the numerical comparison of a flat and a fault-tolerant run shows a
model difference, this isolates one coordinate -- by default the parameter
element with the largest flat-vs-shift difference after ``--step`` -- and
recomputes, in fp64, the AdamW recurrence of each run from its dumps of steps
k-1 and k (``--reference-dump``): m_k = b1 m + (1 - b1) g, v_k = b2 v +
(1 - b2) g^2 and the decoupled-decay update of the fp32 master weight.  The
residuals (observed - recomputed) show whether a run's optimizer followed the
formula on that coordinate, and the cross-run differences of g, m, v and the
master show where the two runs part.  The reference's single-coordinate
diagnostic (scripts/trace_v1_adam.py) plays the same role; one coordinate
does not establish a global cause.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import torch


def _load(run, step, rank):
    return torch.load(Path(run) / f"reference_step{step}_r{rank}.pt", map_location="cpu", weights_only=False)


def _param_id(dump, name):
    return list(dump["offsets"]).index(name) if "offsets" in dump else list(dump["model"]).index(name)


def _at(t, index):
    return float(t.detach().reshape(-1)[index].double())


def trace(prev, cur, name, index) -> dict:
    pid = _param_id(cur, name)
    sp, sc = prev["optimizer"]["state"][pid], cur["optimizer"]["state"][pid]
    grp = prev["optimizer"]["param_groups"][0]
    b1, b2 = (float(x) for x in grp["betas"])
    lr, eps, wd = float(grp["lr"]), float(grp["eps"]), float(grp["weight_decay"])
    t = int(float(sc["step"]))
    off = cur["offsets"][name][0]
    g = float(cur["gradients"].reshape(-1)[off + index].double())
    m0, v0, w0 = _at(sp["exp_avg"], index), _at(sp["exp_avg_sq"], index), _at(sp["master"], index)
    m1, v1, w1 = _at(sc["exp_avg"], index), _at(sc["exp_avg_sq"], index), _at(sc["master"], index)
    m_pred = b1 * m0 + (1 - b1) * g
    v_pred = b2 * v0 + (1 - b2) * g * g

    def update(m, v):
        return w0 * (1 - lr * wd) - lr * (m / (1 - b1 ** t)) / (math.sqrt(v / (1 - b2 ** t)) + eps)

    return {"adam_step": t, "lr": lr, "betas": [b1, b2], "eps": eps, "weight_decay": wd,
            "g": g, "m_prev": m0, "m": m1, "m_pred": m_pred, "m_residual": m1 - m_pred,
            "v_prev": v0, "v": v1, "v_pred": v_pred, "v_residual": v1 - v_pred,
            "master_prev": w0, "master": w1, "master_pred_from_observed_moments": update(m1, v1),
            "master_pred_from_recurrence": update(m_pred, v_pred), "master_residual": w1 - update(m1, v1),
            "param_bf16": _at(cur["model"][name], index)}


def worst_coordinate(flat_dump, shift_dump) -> tuple[str, int, float]:
    best = ("", 0, -1.0)
    for name, a in flat_dump["model"].items():
        d = (a.float() - shift_dump["model"][name].float()).abs().reshape(-1)
        if d.numel() == 0:
            continue
        i = int(torch.argmax(d))
        if float(d[i]) > best[2]:
            best = (name, i, float(d[i]))
    # no model difference: the largest master-weight difference instead
    if best[2] <= 0.0:
        for pid, name in enumerate(flat_dump["offsets"]):
            a = flat_dump["optimizer"]["state"][pid]["master"]
            d = (a - shift_dump["optimizer"]["state"][pid]["master"]).abs().reshape(-1)
            if d.numel() and float(d.max()) > best[2]:
                i = int(torch.argmax(d))
                best = (name, i, float(d[i]))
    return best


def compare(flat_dir, shift_dir, step, rank=0, name=None, index=None) -> dict:
    fp, fc = _load(flat_dir, step - 1, rank), _load(flat_dir, step, rank)
    sp, sc = _load(shift_dir, step - 1, rank), _load(shift_dir, step, rank)
    diff = None
    if name is None:
        name, index, diff = worst_coordinate(fc, sc)
    f, s = trace(fp, fc, name, index), trace(sp, sc, name, index)
    keys = ("g", "m_prev", "m", "v_prev", "v", "master_prev", "master", "param_bf16")
    return {"selected": {"step": step, "rank": rank, "parameter": name, "index": index, "max_abs_difference": diff},
            "flat": f, "shift": s, "cross_run_differences": {k: f[k] - s[k] for k in keys},
            "note": "fp64 recomputation from fp32 dumps; residuals include the fp32 rounding of the update"}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("flat_dir")
    ap.add_argument("shift_dir")
    ap.add_argument("--step", type=int, required=True)
    ap.add_argument("--rank", type=int, default=0)
    ap.add_argument("--param", default=None)
    ap.add_argument("--index", type=int, default=None)
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    rep = compare(a.flat_dir, a.shift_dir, a.step, a.rank, a.param, a.index)
    text = json.dumps(rep, indent=1, sort_keys=True)
    if a.out:
        Path(a.out).write_text(text)
    print(text)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
