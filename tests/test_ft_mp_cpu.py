"""Unplanned fault in a model-parallel replica on CPU/gloo: 2 DP replicas x
(TP2 x PP2) of the tiny MoE under supervisors and the C++ lighthouse.  One TP
rank of replica 0 SIGKILLs itself mid-backward at step 5; the launcher stops
the rest of the replica, replica 1 continues alone, replica 0 is relaunched
(with a different device placement: stage migration), every rank heals from
the same-coordinate rank of replica 1, and the replicas commit jointly with
equal state hashes again."""
import json
import socket

import pytest

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


@pytest.mark.parametrize("inject", ["sigkill_bwd@5", "sigkill_step@5"])
def test_tp_rank_sigkill_recovers_with_migration(tmp_path, inject):
    """sigkill_bwd: the rank dies mid-backward (CPU only); sigkill_step: the
    form used on GPUs -- the rank dies between steps and the rest of its
    replica stops at the same boundary on the host."""
    lh, mp, sp_ = _ports(3)
    cfg = {
        "entry_module": "shift_b200.ft.mp_train",
        "nproc_per_node": 4,
        "train_args": ["--model", "tiny", "--device", "cpu", "--seq-len", "128", "--batch", "1", "--microbatches",
                       "2", "--tp", "2", "--pp", "2", "--audit-state", "--hash-every", "1", "--data", "random",
                       "--communication-timeout", "20", "--inject", inject, "--inject-rank", "1",
                       "--inject-replica", "0"],
        "lighthouse_port": lh, "master_port": mp, "store_port_base": sp_ + 1000 if sp_ < 60000 else 20000,
        "min_replicas": 1, "heartbeat_timeout_ms": 400, "join_timeout_ms": 300, "quorum_tick_ms": 20,
        "target_steps": 1000,
        # placement labels only on CPU: the relaunch moves every rank to "spare" devices
        "devices": [[0, 1, 2, 3], [4, 5, 6, 7]], "restart_devices": [[8, 9, 10, 11], [4, 5, 6, 7]],
    }
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "mp", cpath, replicas=2, seconds=900)
    s.start(timeout=300)
    try:
        rec = s.unplanned_fault(0, timeout=300)
        assert rec["restored_hashes_match"]
        assert rec["killed_stage"] == 0 and rec["killed_tp_rank"] == 1
        assert rec["placement_before"] != rec["placement_after"]
        s.await_(lambda: s.last_step(0) >= rec["joint_step"] + 3, 300, "3 joint commits")
    finally:
        s.finish()
    # after recovery both replicas commit the same states at the same steps, on every rank
    rows = [r for r in s.reader.all_rows if r["kind"] == "commit" and r.get("hashes")]
    by = {}
    for r in rows:
        if r["step"] > rec["joint_step"]:
            by.setdefault((r["step"], r["rank"]), {})[r["rid"]] = r["hashes"]
    joint = [v for v in by.values() if len(v) == 2]
    assert joint, "no joint commits with hashes after recovery"
    for v in joint:
        for k in ("model", "optimizer", "scheduler"):
            assert v[0][k] == v[1][k]


def test_pp_stage_sigkill_recovers_with_stages_swapped(tmp_path):
    """The 4-GPU form of the scenario: replicas of PP2 without tensor
    parallelism; stage 0 of replica 0 dies between steps and the replica is
    relaunched with its two stages swapped between its own devices."""
    lh, mp, sp_ = _ports(3)
    cfg = {
        "entry_module": "shift_b200.ft.mp_train",
        "nproc_per_node": 2,
        "train_args": ["--model", "tiny", "--device", "cpu", "--seq-len", "128", "--batch", "1", "--microbatches",
                       "2", "--tp", "1", "--pp", "2", "--audit-state", "--hash-every", "1", "--data", "random",
                       "--communication-timeout", "20", "--inject", "sigkill_step@5", "--inject-rank", "0",
                       "--inject-replica", "0"],
        "lighthouse_port": lh, "master_port": mp, "store_port_base": sp_ + 1000 if sp_ < 60000 else 20000,
        "min_replicas": 1, "heartbeat_timeout_ms": 400, "join_timeout_ms": 300, "quorum_tick_ms": 20,
        "target_steps": 1000,
        "devices": [[0, 1], [2, 3]], "restart_devices": [[1, 0], [2, 3]],
    }
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "pp", cpath, replicas=2, seconds=900)
    s.start(timeout=300)
    try:
        rec = s.unplanned_fault(0, timeout=300)
        assert rec["restored_hashes_match"]
        assert rec["killed_stage"] == 0
        assert rec["placement_before"] != rec["placement_after"]
        s.await_(lambda: s.last_step(0) >= rec["joint_step"] + 3, 300, "3 joint commits")
    finally:
        s.finish()
