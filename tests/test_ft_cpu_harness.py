"""End-to-end fault tolerance on CPU/gloo: the tiny Qwen-style MoE as 2 DP
replicas x 1 process under supervisors and the C++ lighthouse.  Replica 1 is
SIGKILLed at step 5, the survivor commits alone, replica 1 is relaunched, heals
from the survivor's live state and the joint state audit passes."""
import json
import socket

from shift_b200.analysis.verify import verify
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


def test_kill_at_step_5_heal_and_audit(tmp_path):
    lh, mp, sp_ = _ports(3)
    cfg = {
        "train_args": ["--model", "tiny", "--device", "cpu", "--seq-len", "128", "--batch", "4", "--audit-state",
                       "--hash-every", "1", "--data", "random", "--communication-timeout", "20"],
        "lighthouse_port": lh, "master_port": mp, "store_port_base": sp_ + 1000 if sp_ < 60000 else 20000,
        "min_replicas": 1, "heartbeat_timeout_ms": 400, "join_timeout_ms": 300, "quorum_tick_ms": 20,
        "target_steps": 1000,
    }
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "tiny", cpath, replicas=2, seconds=600)
    s.start(timeout=120)
    try:
        s.await_(lambda: s.last_step(1) >= 5, 120, "step 5")
        rec = s.fault(1, "launcher", timeout=120)
        assert rec["restored_hashes_match"]
        s.await_(lambda: s.last_step(1) >= rec["joint_step"] + 3, 120, "3 joint commits")
    finally:
        s.finish()
    res = verify(tmp_path / "tiny", replicas=2, ranks=1)
    failed = {k: v for k, v in res["checks"].items() if not v["pass"]}
    assert res["pass"], failed
    from shift_b200.analysis.latency import summarize
    lat = summarize(tmp_path / "tiny")
    assert lat["faults"] == 1 and lat["fault_to_joint_s"]["median"] > 0
    assert lat["commit_intervals"]["0"]["commits"] > 5
