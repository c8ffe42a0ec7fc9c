"""The model-free probe (one large parameter) under the same supervisors:
quorum + cross-replica average + AdamW per step, and a kill / heal of one
replica restores the 1-parameter state bit-exactly.  Also the resource
snapshot of the session's processes."""
import json
import socket

from shift_b200.control.resource_probe import snapshot
from shift_b200.control.session import Session


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


def test_native_probe_kill_heal(tmp_path):
    lh, mp, spb = _ports(3)
    cfg = {"entry_module": "shift_b200.ft.native_probe",
           "train_args": ["--numel", "200000", "--device", "cpu", "--audit-state", "--hash-every", "1",
                          "--communication-timeout", "20"],
           "lighthouse_port": lh, "master_port": mp, "store_port_base": spb + 1000 if spb < 60000 else 20000,
           "min_replicas": 1, "heartbeat_timeout_ms": 400, "join_timeout_ms": 300, "quorum_tick_ms": 20}
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "probe", cpath, replicas=2, seconds=300)
    s.start(timeout=120)
    try:
        s.await_(lambda: s.last_step(1) >= 5, 120, "step 5")
        snap = snapshot(s.dir)
        assert snap["processes"] and snap["total_rss_kib"] > 0
        rec = s.fault(1, "launcher", timeout=120)
        assert rec["restored_hashes_match"]
        s.await_(lambda: s.last_step(1) >= rec["joint_step"] + 2, 120, "joint commits")
    finally:
        s.finish()
    commits = [r for r in s.reader.all_rows if r["kind"] == "commit" and r["rid"] == 0]
    assert all("reduce_seconds" in c and "optimizer_seconds" in c for c in commits)
    ready = [r for r in s.reader.all_rows if r["kind"] == "ready" and r.get("probe")]
    assert ready and ready[0]["state_bytes"] == 200000 * (4 + 12)
