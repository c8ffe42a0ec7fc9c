"""C++ lighthouse + replica manager server: quorum formation, heal
assignment, commit vote, heartbeat expiry (host processes only)."""
import threading
import time

import pytest

from shift_b200.ft.native import (LighthouseClient, LighthouseServer, ManagerClient, ManagerServerHandle,
                                  spawn_lighthouse)


def _quorum_threads(fns):
    out = [None] * len(fns)
    errs = []

    def run(i, f):
        try:
            out[i] = f()
        except Exception as e:  # pragma: no cover - surfaced below
            errs.append(e)

    ts = [threading.Thread(target=run, args=(i, f)) for i, f in enumerate(fns)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(30)
    assert not errs, errs
    return out


def test_quorum_forms_without_waiting_for_tick_and_assigns_heal():
    lh = LighthouseServer(min_replicas=1, join_timeout_ms=5000, heartbeat_timeout_ms=2000, quorum_tick_ms=1000)
    try:
        m0 = ManagerServerHandle("shift0", lh.address, 1, "127.0.0.1:1111")
        m1 = ManagerServerHandle("shift1", lh.address, 1, "127.0.0.1:2222")
        c0, c1 = ManagerClient(m0.address, 0), ManagerClient(m1.address, 0)
        time.sleep(0.3)  # both heartbeating
        t0 = time.monotonic()
        r0, r1 = _quorum_threads([lambda: c0.quorum(7, "meta0"), lambda: c1.quorum(3, "meta1")])
        elapsed = time.monotonic() - t0
        # event driven: all live replicas asked -> no join timeout, no tick wait
        assert elapsed < 0.5, elapsed
        assert r0.quorum_id == r1.quorum_id == 1
        assert (r0.replica_rank, r1.replica_rank) == (0, 1)
        assert r0.replica_world_size == 2 and r0.max_step == 7
        assert not r0.heal and r1.heal
        assert r1.recover_src_manager_address == m0.address and r1.recover_src_replica_rank == 0
        assert r0.recover_dst_replica_ranks == [1]
        assert r0.store_address == "127.0.0.1:1111" == r1.store_address
        assert c1.checkpoint_metadata(m0.address, 0) == "meta0"
        # same membership -> same quorum id
        r0b, r1b = _quorum_threads([lambda: c0.quorum(8), lambda: c1.quorum(8)])
        assert r0b.quorum_id == 1 and not r1b.heal
        # commit vote of a 1-rank replica
        assert c0.should_commit(8, True) is True
        assert c1.should_commit(8, False) is False
        for c in (c0, c1):
            c.close()
        m0.stop()
        m1.stop()
    finally:
        lh.stop()


def test_dead_replica_does_not_block_after_heartbeat_timeout():
    lh = LighthouseServer(min_replicas=1, join_timeout_ms=60_000, heartbeat_timeout_ms=300, quorum_tick_ms=20)
    try:
        m0 = ManagerServerHandle("a", lh.address, 1, "s0")
        m1 = ManagerServerHandle("b", lh.address, 1, "s1")
        c0 = ManagerClient(m0.address, 0)
        time.sleep(0.2)
        m1.stop()  # replica b dies: heartbeats stop
        t0 = time.monotonic()
        r = c0.quorum(1)
        assert time.monotonic() - t0 < 2.0
        assert r.replica_world_size == 1 and r.members == [("a", 1)]
        c0.close()
        m0.stop()
    finally:
        lh.stop()


def test_manager_aggregates_local_ranks_and_votes():
    lh = LighthouseServer(min_replicas=1, join_timeout_ms=1000, heartbeat_timeout_ms=1000, quorum_tick_ms=20)
    try:
        m = ManagerServerHandle("r0", lh.address, 2, "st")
        cs = [ManagerClient(m.address, r) for r in range(2)]
        res = _quorum_threads([lambda c=c: c.quorum(4) for c in cs])
        assert res[0].quorum_id == res[1].quorum_id and res[0].replica_world_size == 1
        votes = _quorum_threads([lambda: cs[0].should_commit(4, True), lambda: cs[1].should_commit(4, False)])
        assert votes == [False, False]
        votes = _quorum_threads([lambda: cs[0].should_commit(5, True), lambda: cs[1].should_commit(5, True)])
        assert votes == [True, True]
        for c in cs:
            c.close()
        m.stop()
    finally:
        lh.stop()


def test_min_replicas_and_join_timeout():
    lh = LighthouseServer(min_replicas=2, join_timeout_ms=200, heartbeat_timeout_ms=5000, quorum_tick_ms=20)
    try:
        a = LighthouseClient(lh.address)
        b = LighthouseClient(lh.address)
        got = {}

        def qa():
            got["a"] = a.quorum("a", 1)

        t = threading.Thread(target=qa)
        t.start()
        time.sleep(0.4)
        assert "a" not in got  # below min_replicas: keeps waiting past the join timeout
        got["b"] = b.quorum("b", 1)
        t.join(5)
        assert got["a"][0] == got["b"][0] == 1
        assert [m["replica_id"] for m in got["a"][1]] == ["a", "b"]
        st = a.status()
        assert st["formed"] == 1
    finally:
        lh.stop()


def test_standalone_daemon():
    p, addr = spawn_lighthouse(min_replicas=1)
    try:
        c = LighthouseClient(addr)
        qid, mem = c.quorum("solo", 0)
        assert qid == 1 and mem[0]["replica_id"] == "solo"
        c.close()
    finally:
        p.terminate()
        p.wait(5)


def test_timeout_quorum_waits_for_a_live_replica_that_is_ahead():
    """A relaunched replica (step 0) must not form a quorum of its own on the
    join timeout while a live replica ahead of it is between requests: it
    waits and heals from that replica (bounded)."""
    lh = LighthouseServer(min_replicas=1, join_timeout_ms=100, heartbeat_timeout_ms=2000, quorum_tick_ms=10)
    try:
        a, b = LighthouseClient(lh.address), LighthouseClient(lh.address)
        _, ma = a.quorum("A", 20)              # A trains alone at step 20
        assert [m["replica_id"] for m in ma] == ["A"]
        a.heartbeat("A")
        res = {}
        th = threading.Thread(target=lambda: res.setdefault("b", b.quorum("B", 0)))
        t0 = time.monotonic()
        th.start()
        time.sleep(0.6)                        # far past the join timeout
        assert "b" not in res, "B formed a quorum without the live replica ahead of it"
        a.heartbeat("A")
        _, ma2 = a.quorum("A", 21)
        th.join(10)
        waited = time.monotonic() - t0
        assert waited >= 0.6
        ids = sorted(m["replica_id"] for m in res["b"][1])
        assert ids == ["A", "B"] and sorted(m["replica_id"] for m in ma2) == ["A", "B"]
        a.close()
        b.close()
    finally:
        lh.stop()
