"""Process-tree utilities for supervisors: child subreaper, descendant
discovery from /proc, tree termination, and orphan reaping that never steals
the exit status of a child owned by a ``subprocess.Popen``.

Same contract as shift_full/process_tree.py:37-97 and shift_min/supervisor.py:12-33:
a supervisor adopts orphaned grandchildren and collects only zombies among
its direct children that are not excluded.  Process state comes from
``/proc/<pid>/status``.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import os
import signal
import sys
import time

_PR_SET_CHILD_SUBREAPER = 36       # <linux/prctl.h>
_PR_GET_CHILD_SUBREAPER = 37


class _Libc:
    """Lazily bound ``prctl(2)`` from the C library of this process."""

    fn = None

    @classmethod
    def prctl(cls, option: int, value: int) -> int:
        if sys.platform != "linux":
            raise RuntimeError(f"prctl is Linux-only (this is {sys.platform})")
        if cls.fn is None:
            libc = ctypes.CDLL(ctypes.util.find_library("c") or None, use_errno=True)
            f = libc.prctl
            f.restype = ctypes.c_int
            f.argtypes = [ctypes.c_int] + [ctypes.c_ulong] * 4
            cls.fn = f
        rc = cls.fn(option, value, 0, 0, 0)
        if rc < 0:
            code = ctypes.get_errno()
            raise OSError(code, f"prctl({option}): {os.strerror(code)}")
        return rc


def enable_subreaper():
    """Make this process adopt orphaned descendants (instead of init)."""
    _Libc.prctl(_PR_SET_CHILD_SUBREAPER, 1)


def is_subreaper() -> bool:
    flag = ctypes.c_int(-1)
    _Libc.prctl(_PR_GET_CHILD_SUBREAPER, ctypes.addressof(flag))
    return flag.value != 0


def _status(pid: int):
    """(state letter, parent pid) from /proc/<pid>/status, or None once the
    process is gone or unreadable."""
    fields = {}
    try:
        with open(f"/proc/{pid}/status") as f:
            for line in f:
                key, _, val = line.partition(":")
                if key in ("State", "PPid"):
                    fields[key] = val.strip()
                    if len(fields) == 2:
                        break
    except OSError:
        return None
    try:
        return fields["State"][:1], int(fields["PPid"])
    except (KeyError, ValueError):
        return None


def _all_pids():
    with os.scandir("/proc") as it:
        return [int(e.name) for e in it if e.name.isdigit()]


def children_of(parent: int):
    """[(pid, state letter)] of the live or zombie children of ``parent``."""
    out = []
    for pid in _all_pids():
        st = _status(pid)
        if st is not None and st[1] == parent:
            out.append((pid, st[0]))
    return out


def descendants(root: int) -> list[int]:
    """All live descendants of ``root`` (breadth first), excluding root."""
    parent_of = {}
    for pid in _all_pids():
        st = _status(pid)
        if st is not None:
            parent_of[pid] = st[1]
    kids: dict[int, list[int]] = {}
    for pid, pp in parent_of.items():
        kids.setdefault(pp, []).append(pid)
    out, frontier = [], [root]
    while frontier:
        nxt = []
        for p in frontier:
            for c in kids.get(p, []):
                out.append(c)
                nxt.append(c)
        frontier = nxt
    return out


def terminate(proc_or_pid, sig=signal.SIGKILL) -> list[int]:
    """Signal a process and all of its descendants (leaves first)."""
    pid = proc_or_pid if isinstance(proc_or_pid, int) else proc_or_pid.pid
    victims = descendants(pid)
    for p in reversed(victims):
        try:
            os.kill(p, sig)
        except ProcessLookupError:
            pass
    try:
        os.kill(pid, sig)
    except ProcessLookupError:
        pass
    return [pid] + victims


def reap_orphans(exclude_pids=(), timeout: float = 2.0) -> list[int]:
    """Collect adopted orphans: wait, by pid, for each zombie child of this
    process that is not in ``exclude_pids``, until no such child is left or
    ``timeout`` seconds have passed.  A child owned by a ``subprocess.Popen``
    belongs in ``exclude_pids``; waiting by pid (never ``waitpid(-1)``) keeps
    its exit status for its owner."""
    if not is_subreaper():
        raise RuntimeError("reap_orphans needs enable_subreaper() first: orphans are not re-parented here")
    keep = {int(p) for p in exclude_pids}
    me = os.getpid()
    give_up = time.monotonic() + max(0.0, timeout)
    nap = 0.001
    collected: list[int] = []
    while True:
        left = [(pid, st) for pid, st in children_of(me) if pid not in keep]
        for pid, st in left:
            if st != "Z":
                continue
            try:
                got, _ = os.waitpid(pid, os.WNOHANG)
            except ChildProcessError:       # somebody else collected it
                got = 0
            if got == pid:
                collected.append(pid)
        remaining = give_up - time.monotonic()
        if not left or remaining <= 0:
            return collected
        time.sleep(min(nap, remaining))
        nap = min(nap * 2, 0.05)
