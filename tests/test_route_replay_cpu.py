"""Route replay from a common anchor: a flat run and a fault-tolerant run
(2 replicas) both continue from the flat run's step-2 dump
(--reference-anchor); starting from identical bits, the next step has the
same initial-state digests, batch plan and per-layer routing, and the
step-3 dumps agree within the numerical tolerances."""
import json
import socket
import subprocess as sp
import sys
from pathlib import Path

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


def test_anchored_route_replay(tmp_path):
    base = ["--model", "tiny", "--device", "cpu", "--seq-len", "64", "--batch", "2", "--data", "random",
            "--communication-timeout", "20"]

    def flat(session, steps, extra):
        sp.run([sys.executable, "-m", "shift_b200.ft.train", "--session", session, "--replica", "0", "--root",
                str(tmp_path), "--lighthouse", "127.0.0.1:1", "--mode", "flat", "--steps", str(steps), *base, *extra],
               check=True, cwd=ROOT, timeout=300)

    flat("anchor", 2, ["--reference-dump", "2"])
    anchor = ["--reference-anchor", str(tmp_path / "anchor"), "--reference-anchor-step", "2",
              "--trace-routing", "--audit-state", "--reference-dump", "3"]
    flat("flat", 3, anchor)
    lh, mp, spb = _ports(3)
    cfg = {"train_args": base + anchor, "lighthouse_port": lh, "master_port": mp,
           "store_port_base": spb + 1000 if spb < 60000 else 20000, "min_replicas": 2,
           "heartbeat_timeout_ms": 1000, "join_timeout_ms": 1000, "quorum_tick_ms": 20, "target_steps": 3}
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "shift", cpath, replicas=2, seconds=300)
    s.start(timeout=200)
    try:
        s.await_(lambda: all(s.last_step(r) >= 3 for r in (0, 1)), 200, "step 3")
    finally:
        s.finish()
    rep = summarize(tmp_path / "flat", tmp_path / "shift")
    assert rep["pass"], json.dumps(rep, default=str)[:3000]
    assert rep["checks"]["step_coverage"]["flat_steps"] == [2]
    assert rep["checks"]["same_routing"]["keys"] == 2 * 2          # samples x MoE layers of step 2
