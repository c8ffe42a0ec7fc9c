"""PeerWatch: a member that dies without farewell trips the status word at
once; a member that leaves on purpose, or a process outside the quorum, does
not.  Host-side only (the child processes are killed on the host; no GPU)."""
import multiprocessing as mp
import os
import signal
import time

from shift_b200.ft.peer_watch import PeerWatch


def _child(conn, graceful):
    w = PeerWatch("child", None)
    conn.send(w.address)
    conn.recv()                      # wait for the parent to connect (or for the order to leave)
    if graceful:
        w.close()
        conn.send("closed")
    time.sleep(60)


def _spawn(graceful=False):
    ctx = mp.get_context("spawn")
    a, b = ctx.Pipe()
    p = ctx.Process(target=_child, args=(b, graceful), daemon=True)
    p.start()
    return p, a, a.recv()


def _wait(cond, limit=10.0):
    end = time.monotonic() + limit
    while not cond() and time.monotonic() < end:
        time.sleep(0.005)
    return cond()


def test_sigkill_of_a_member_trips_within_a_second():
    events = []
    w = PeerWatch("me", None, event=lambda k, **f: events.append((k, f)))
    p, conn, addr = _spawn()
    try:
        w.set_members({"child": addr})
        conn.send("go")
        time.sleep(0.05)
        t0 = time.monotonic()
        os.kill(p.pid, signal.SIGKILL)
        assert _wait(lambda: w.tripped == 1)
        assert time.monotonic() - t0 < 1.0
        assert "child" in w.dead
        assert events and events[-1][0] == "peer_dead" and events[-1][1]["member"] is True
        # a later step re-trips while the dead member is still in the quorum ...
        assert w.check() and w.tripped == 2
        # ... and not once the quorum has dropped it
        w.set_members({})
        assert not w.check() and w.tripped == 2
    finally:
        p.join(5)
        w.close()


def test_farewell_does_not_trip():
    events = []
    w = PeerWatch("me", None, event=lambda k, **f: events.append((k, f)))
    p, conn, addr = _spawn(graceful=True)
    try:
        w.set_members({"child": addr})
        conn.send("go")
        assert conn.recv() == "closed"
        assert _wait(lambda: any(k == "peer_left" for k, _ in events))
        os.kill(p.pid, signal.SIGKILL)
        time.sleep(0.2)
        assert w.tripped == 0 and not w.dead
    finally:
        p.join(5)
        w.close()


def test_death_outside_the_quorum_is_recorded_not_tripped():
    w = PeerWatch("me", None)
    p, conn, addr = _spawn()
    try:
        w.set_members({"child": addr})
        conn.send("go")
        time.sleep(0.05)
        w.set_members({})            # the quorum moved on before the process died
        os.kill(p.pid, signal.SIGKILL)
        assert _wait(lambda: "child" in w.dead)
        assert w.tripped == 0
    finally:
        p.join(5)
        w.close()
