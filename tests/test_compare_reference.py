"""Numerical oracle on CPU: the flat baseline (one process, whole global
batch, no Manager) and the fault-tolerant run (2 replicas, quorum, group
average) agree per step within the reference's tolerances; a perturbed run
does not.  The trajectory summary of the same two runs finds the same initial
state, batch plans and per-layer routing; a tampered routing row fails it."""
import json
import socket
import subprocess as sp
import sys
from pathlib import Path

import torch

from shift_b200.analysis.compare_reference import compare_runs
from shift_b200.analysis.trajectory import summarize
from shift_b200.control.session import Session

ROOT = Path(__file__).resolve().parents[1]


def _ports(n):
    socks, out = [], []
    for _ in range(n):
        s = socket.socket()
        s.bind(("127.0.0.1", 0))
        socks.append(s)
        out.append(s.getsockname()[1])
    for s in socks:
        s.close()
    return out


def test_flat_vs_shift_reference_dumps(tmp_path):
    common = ["--model", "tiny", "--device", "cpu", "--seq-len", "64", "--batch", "2", "--data", "random",
              "--reference-dump", "1,2,3", "--communication-timeout", "20", "--audit-state", "--trace-routing", "--profile-timings"]
    flat_dir = tmp_path / "flat"
    sp.run([sys.executable, "-m", "shift_b200.ft.train", "--session", "flat", "--replica", "0", "--root",
            str(tmp_path), "--lighthouse", "127.0.0.1:1", "--mode", "flat", "--steps", "3", *common],
           check=True, cwd=ROOT, timeout=300)
    lh, mp, spb = _ports(3)
    cfg = {"train_args": common, "lighthouse_port": lh, "master_port": mp,
           "store_port_base": spb + 1000 if spb < 60000 else 20000, "min_replicas": 2,
           "heartbeat_timeout_ms": 1000, "join_timeout_ms": 1000, "quorum_tick_ms": 20, "target_steps": 3}
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "shift", cpath, replicas=2, seconds=300)
    s.start(timeout=200)
    try:
        s.await_(lambda: all(s.last_step(r) >= 3 for r in (0, 1)), 200, "3 steps")
    finally:
        s.finish()
    res = compare_runs(flat_dir, tmp_path / "shift", steps=[1, 2, 3])
    assert res["pass"], json.dumps(res, default=str)[:2000]
    # strict (bitwise) comparison: the runs round their reductions in different orders
    strict = compare_runs(flat_dir, tmp_path / "shift", steps=[1, 2, 3], strict=True)
    assert strict["strict"] and strict["tolerances"]["model"] == (0.0, 0.0)
    assert all(strict["steps"][f"{k}/0"]["scheduler"]["pass"] for k in (1, 2, 3))
    assert not strict["pass"]          # different reduction orders differ in the last bits
    # a run compared with itself passes strict mode
    assert compare_runs(flat_dir, flat_dir, steps=[1, 2, 3], strict=True)["pass"]
    commits = [json.loads(x) for f in sorted((tmp_path / "shift").glob("events_g0_r*.jsonl"))
               for x in f.read_text().splitlines() if '"commit"' in x]
    commits = [c for c in commits if c.get("kind") == "commit"]
    assert commits and all(c["schedule_seconds"] >= 0 and c["gradient_check_seconds"] >= 0 and
                           {"d2h_seconds", "dispatch_seconds", "wait_seconds", "cross_host_seconds"} <= c.keys()
                           for c in commits)
    traj = summarize(flat_dir, tmp_path / "shift", comparison=res)
    assert traj["pass"], json.dumps(traj, default=str)[:3000]
    assert traj["checks"]["same_routing"]["keys"] == 3 * 2 * 2     # steps x samples x MoE layers
    # a routing digest that differs is caught
    ev = sorted(flat_dir.glob("events_g0_r*.jsonl"))[0]
    rows = [json.loads(x) for x in ev.read_text().splitlines() if x.strip()]
    for r in rows:
        if r.get("kind") == "routing":
            r["topk_hash"] = "0" * 64
            break
    ev.write_text("".join(json.dumps(r, sort_keys=True) + "\n" for r in rows))
    bad = summarize(flat_dir, tmp_path / "shift", comparison=res)
    assert not bad["pass"] and not bad["checks"]["same_routing"]["pass"]
    assert bad["checks"]["same_batch_plans"]["pass"]
    # single-coordinate AdamW trace: both runs follow the recurrence on the coordinate where they differ most
    from shift_b200.analysis.adam_trace import compare as adam_compare
    tr = adam_compare(flat_dir, tmp_path / "shift", step=3)
    for run in ("flat", "shift"):
        t = tr[run]
        assert t["adam_step"] == 3
        assert abs(t["m_residual"]) <= 1e-6 * max(1.0, abs(t["m"])) + 1e-9, t
        assert abs(t["v_residual"]) <= 1e-5 * abs(t["v"]) + 1e-12, t
        assert abs(t["master_residual"]) <= 1e-6 * max(1.0, abs(t["master"])), t
    # the oracle is sensitive: a perturbed model fails it
    p = torch.load(flat_dir / "reference_step3_r0.pt", weights_only=False)
    name = next(iter(p["model"]))
    p["model"][name] = p["model"][name] + 1e-3
    torch.save(p, flat_dir / "reference_step3_r0.pt")
    assert not compare_runs(flat_dir, tmp_path / "shift", steps=[3])["pass"]


def test_strict_mode_sees_what_tolerances_forgive(tmp_path):
    """Dumps differing by one ulp, by dtype, by the sign of zero, or in an int
    leaf pass the tolerant comparison and fail the strict one."""
    base = {"gradients": {"w": torch.tensor([1.0, 0.0, 2.0])},
            "model": {"w": torch.tensor([1.0, 0.0, 2.0])},
            "optimizer": {"state": {0: {"step": 3, "exp_avg": torch.tensor([0.5, 0.25])}}},
            "scheduler": {"last_epoch": 3}}
    import copy
    variants = {
        "ulp": lambda d: d["model"].__setitem__("w", torch.nextafter(d["model"]["w"], torch.tensor(9.0))),
        "dtype": lambda d: d["gradients"].__setitem__("w", d["gradients"]["w"].double()),
        "negzero": lambda d: d["model"].__setitem__("w", torch.tensor([1.0, -0.0, 2.0])),
        "int_leaf": lambda d: d["optimizer"]["state"][0].__setitem__("step", 4),
    }
    a = tmp_path / "a"
    a.mkdir()
    torch.save(base, a / "reference_step1_r0.pt")
    for name, change in variants.items():
        b = tmp_path / name
        b.mkdir()
        d = copy.deepcopy(base)
        change(d)
        torch.save(d, b / "reference_step1_r0.pt")
        assert not compare_runs(a, b, steps=[1], strict=True)["pass"], name
        if name != "int_leaf":       # the tolerant mode compares tensors only
            assert compare_runs(a, b, steps=[1])["pass"], name
    assert compare_runs(a, a, steps=[1], strict=True)["pass"]
