"""v1 fail-stop rotation on CPU/gloo (tiny MoE, 2 replicas x 1 process):
seeded victims, a cold restart and a cpu standby activated by the
supervisor, each fault audited for RPO 0 and restore hashes; and the
disk-checkpoint restart scenario (both replicas killed, resumed from disk,
training jointly again)."""
import json
import socket

from shift_b200.control.rotation import Rotation, summarize
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


def _config(tmp_path, extra=(), **keys):
    lh, mp, sp_ = _ports(3)
    cfg = {
        "train_args": ["--model", "tiny", "--device", "cpu", "--seq-len", "64", "--batch", "2", "--audit-state",
                       "--hash-every", "1", "--data", "random", "--communication-timeout", "20", *extra],
        "lighthouse_port": lh, "master_port": mp, "store_port_base": sp_ + 1000 if sp_ < 60000 else 20000,
        "min_replicas": 1, "heartbeat_timeout_ms": 400, "join_timeout_ms": 300, "quorum_tick_ms": 20,
        "target_steps": 100000,
        **keys,
    }
    p = tmp_path / "cfg.json"
    p.write_text(json.dumps(cfg))
    return p


def test_seeded_rotation_cold_then_cpu_standby(tmp_path):
    s = Session(tmp_path, "rot", _config(tmp_path), replicas=2, seconds=900)
    s.start(timeout=180)
    try:
        rot = Rotation(s, "cold", seed=3)
        first = rot.fault(0)
        rot.mode = "cpu"
        second = rot.fault(1)
    finally:
        s.finish()
    for r in (first, second):
        assert r["pass"], r
        assert r["rpo_zero"] and r["restore_hashes_match"] and r["healthy_pids_unchanged"]
        assert r["restored_step"] >= r["committed_before_fault"]
        assert r["fault_to_joint_seconds"] > 0
    assert first["preparation_seconds"] < 1.0                      # cold: nothing prepared ahead
    assert second["standby_resources"] and all(x["mode"] == "cpu" for x in second["standby_resources"])
    # the victims are drawn from the seeded generator
    import random
    g = random.Random(3)
    assert [first["target"], second["target"]] == [g.randrange(2), g.randrange(2)]
    summ = summarize([first, second])
    assert summ["faults"] == 2 and summ["rpo_zero"] == 2 and summ["all_pass"]
    rows = [json.loads(x) for x in (tmp_path / "rot" / f"controller_r{second['target']}.jsonl").read_text().splitlines()]
    assert any(r.get("kind") == "standby_activated" for r in rows)
    assert json.loads((tmp_path / "rot" / "fault_results.json").read_text())[1]["backup_mode"] == "cpu"


def test_checkpoint_restart_resumes_both_replicas(tmp_path):
    s = Session(tmp_path, "ck", _config(tmp_path, ["--checkpoint-step", "3"]), replicas=2, seconds=900)
    s.start(timeout=180)
    try:
        res = Rotation(s).checkpoint_restart(timeout=300)
    finally:
        s.finish()
    assert res["pass"], res
    assert res["checkpoint_step"] == 3 and res["resumed_steps"] == [3]
    assert res["first_joint_step"] > 3


def test_fast_launch_and_lazy_restart_heal(tmp_path):
    """Generations forked from the preloaded supervisor; the relaunched one
    skips the seeded initialisation and must still restore the live state."""
    s = Session(tmp_path, "fast", _config(tmp_path, fast_launch=True, lazy_restart_init=True), replicas=2,
                seconds=900)
    s.start(timeout=180)
    try:
        res = Rotation(s, "cold", seed=1).fault(0)
    finally:
        s.finish()
    assert res["pass"] and res["rpo_zero"] and res["restore_hashes_match"], res
    sup = [json.loads(x) for r in (0, 1) for x in (tmp_path / "fast" / f"supervisor_r{r}.jsonl").read_text().splitlines()]
    assert sum(1 for r in sup if r.get("kind") == "preloaded") == 2
    launched = [r for r in sup if r.get("kind") == "launched" and r.get("generation") == 1]
    assert launched and "--lazy-init" in launched[0]["command"]
