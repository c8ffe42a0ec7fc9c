"""Transparent mode on CPU/gloo: an unmodified PyTorch script as 2 replicas
under the supervisors and the C++ lighthouse.  Replica 1 is SIGKILLed, the
survivor commits alone, replica 1 is relaunched, heals from the survivor's
live parameters and optimizer state (hash-audited) and the replicas then
commit identical states."""
import json
import socket
from pathlib import Path

from shift_b200.control.session import Session

SCRIPT = Path(__file__).parent / "fixtures" / "plain_torch_train.py"


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


def test_unmodified_script_kill_heal_and_joint_hashes(tmp_path):
    lh, mp, sp_ = _ports(3)
    cfg = {"entry_module": "shift_b200.ft.transparent", "train_args": ["--script", str(SCRIPT)],
           "lighthouse_port": lh, "master_port": mp, "store_port_base": sp_ + 1000 if sp_ < 60000 else 20000,
           "min_replicas": 1, "heartbeat_timeout_ms": 400, "join_timeout_ms": 300, "quorum_tick_ms": 20,
           "target_steps": 100000}
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "tr", cpath, replicas=2, seconds=600)
    s.start(timeout=120)
    try:
        s.await_(lambda: s.last_step(1) >= 5, 120, "step 5")
        rec = s.fault(1, "launcher", timeout=120)
        assert rec["restored_hashes_match"]
        s.await_(lambda: s.last_step(1) >= rec["joint_step"] + 3, 120, "3 joint commits")
    finally:
        s.finish()
    rows = [r for r in s.reader.all_rows if r["kind"] == "commit"]
    by_step = {}
    for r in rows:
        if r["step"] > rec["joint_step"] and r["participants"] == 2:
            by_step.setdefault(r["step"], {})[r["rid"]] = r["hashes"]
    joint = [v for v in by_step.values() if len(v) == 2]
    assert joint and all(v[0] == v[1] for v in joint)
    assert any(r["kind"] == "stopped" for r in s.reader.all_rows)
