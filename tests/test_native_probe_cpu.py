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


def test_spare_shadow_and_snapshot_overlap(tmp_path):
    """Three replicas with two participant slots: the spare joins every
    reduction with a zero contribution and ends each step with the same model
    and optimizer digests as the participants; the snapshot copied during the
    step equals the committed state, which the step never wrote."""
    lh, mp, spb = _ports(3)
    cfg = {"entry_module": "shift_b200.ft.native_probe",
           "train_args": ["--numel", "100000", "--device", "cpu", "--audit-state", "--hash-every", "1",
                          "--communication-timeout", "20", "--min-replicas", "2",
                          "--world-size-mode", "fixed_with_spares", "--snapshot-overlap"],
           "lighthouse_port": lh, "master_port": mp, "store_port_base": spb + 1000 if spb < 60000 else 20000,
           "min_replicas": 2, "heartbeat_timeout_ms": 1000, "join_timeout_ms": 1000, "quorum_tick_ms": 20}
    cpath = tmp_path / "cfg.json"
    cpath.write_text(json.dumps(cfg))
    s = Session(tmp_path, "spares", cpath, replicas=3, seconds=300)
    s.start(timeout=120)
    try:
        s.await_(lambda: all(s.last_step(r) >= 4 for r in (0, 1, 2)), 120, "step 4 on every replica")
    finally:
        s.finish()
    from shift_b200.analysis.trajectory import read_events
    rows, errors, _ = read_events(s.dir)
    assert not errors
    commits = [r for r in rows if r["kind"] == "commit" and r.get("step", 0) <= 4]
    assert {r["participants"] for r in commits} == {2}
    spare = {r["rid"] for r in commits if r["contributed"] is False}
    assert len(spare) == 1, spare
    for step in range(1, 5):
        at = [r for r in commits if r["step"] == step]
        assert len({r["rid"] for r in at}) == 3
        assert len({(r["hashes"]["model"], r["hashes"]["optimizer"]) for r in at}) == 1, step
    snaps = [r for r in rows if r["kind"] == "snapshot_overlap"]
    assert snaps and all(r["source_unchanged"] and r["snapshot_equal"] for r in snaps)
    assert snaps[0]["bytes"] >= 100000 * (4 + 12)      # flat buffers are padded to an alignment
