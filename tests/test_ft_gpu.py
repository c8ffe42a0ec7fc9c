"""Fault tolerance on GPUs through the fused peer-memory paths: kill / heal
over CUDA IPC (2 GPUs) and planned handoff P1f / P2 (3 GPUs).  Ranks are
child processes; NVLS is off; waits are bounded."""
import json
import socket

import pytest
import torch

from shift_b200.analysis.verify import verify
from shift_b200.control.planned import PlannedSession
from shift_b200.control.session import Session

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


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


def test_kill_and_heal_over_peer_memory(tmp_path):
    lh, mp, sp_ = _ports(3)
    cfg = {
        "train_args": ["--model", "tiny", "--device", "cuda", "--reduce", "fused", "--seq-len", "128", "--batch", "4",
                       "--audit-state", "--hash-every", "1", "--communication-timeout", "30"],
        "lighthouse_port": lh, "master_port": mp, "store_port_base": 20000 + (sp_ % 20000),
        "min_replicas": 1, "heartbeat_timeout_ms": 500, "join_timeout_ms": 300, "quorum_tick_ms": 20,
        "devices": [[0], [1]], "env": {"NCCL_NVLS_ENABLE": "0"},
    }
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "gpu", cpath, replicas=2, seconds=600)
    s.start(timeout=300)
    try:
        s.await_(lambda: s.last_step(1) >= 5, 180, "step 5")
        rec = s.fault(1, "launcher", timeout=180)
        assert rec["restored_hashes_match"]
        s.await_(lambda: s.last_step(1) >= rec["joint_step"] + 3, 180, "joint commits")
    finally:
        s.finish()
    res = verify(tmp_path / "gpu", replicas=2, ranks=1)
    assert res["pass"], {k: v for k, v in res["checks"].items() if not v["pass"]}


@pytest.mark.parametrize("variant", ["p1f", "p2"])
def test_planned_handoff_on_gpus(tmp_path, variant):
    if torch.cuda.device_count() < 3:
        pytest.skip("needs 3 GPUs (A, B, C)")
    s = PlannedSession(tmp_path, variant, variant=variant, device="cuda", devices={"A": [0], "B": [1], "C": [2]})
    res = s.run(post_steps=3)
    assert res["returncodes"] == {"A": 0, "B": 0, "C": 0}
    assert res["pass"], {k: v for k, v in res["checks"].items() if not v["pass"]}


@pytest.mark.parametrize("variant", ["p1f", "p2"])
def test_rotation_cycles_on_gpus(tmp_path, variant):
    """Three consecutive B/C rotation rounds on three GPUs (the spare of each
    round is relaunched on the GPU the retired donor left)."""
    if torch.cuda.device_count() < 3:
        pytest.skip("needs 3 GPUs (A, B, C)")
    s = PlannedSession(tmp_path, f"rot_{variant}", variant=variant, device="cuda",
                       devices={"A": [0], "B": [1], "C": [2]})
    res = s.run_cycles(cycles=3, post_steps=6)
    assert res["pass"], {k: v for k, v in res["checks"].items() if not v["pass"]}
    assert all(rc == 0 for rc in res["returncodes"].values()), res["returncodes"]
