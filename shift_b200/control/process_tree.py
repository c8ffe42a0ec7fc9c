"""Process-tree utilities for supervisors: child subreaper, descendant
discovery from /proc, tree termination, and orphan reaping that never steals
the exit status of a child owned by a ``subprocess.Popen``.

Same contract as shift_full/process_tree.py:37-97 and shift_min/supervisor.py:12-33
(a supervisor adopts orphaned grandchildren, reaps only zombies among its
direct children, and only those not excluded).
"""
from __future__ import annotations

import ctypes
import os
import signal
import sys
import time
from pathlib import Path

PR_SET_CHILD_SUBREAPER = 36
PR_GET_CHILD_SUBREAPER = 37
_prctl = None


def _libc_prctl():
    global _prctl
    if not sys.platform.startswith("linux"):
        raise RuntimeError("child subreapers are supported only on Linux")
    if _prctl is None:
        fn = ctypes.CDLL(None, use_errno=True).prctl
        fn.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.c_ulong, ctypes.c_ulong, ctypes.c_ulong]
        fn.restype = ctypes.c_int
        _prctl = fn
    return _prctl


def _prctl_call(option: int, arg) -> int:
    fn = _libc_prctl()
    ctypes.set_errno(0)
    ptr = ctypes.c_void_p(arg) if isinstance(arg, int) else ctypes.cast(arg, ctypes.c_void_p)
    r = fn(option, ptr, 0, 0, 0)
    if r == -1:
        err = ctypes.get_errno()
        raise OSError(err, os.strerror(err))
    return r


def enable_subreaper():
    _prctl_call(PR_SET_CHILD_SUBREAPER, 1)


def is_subreaper() -> bool:
    v = ctypes.c_int(0)
    _prctl_call(PR_GET_CHILD_SUBREAPER, ctypes.byref(v))
    return v.value == 1


def _proc_stat(pid: int):
    """(state, ppid) of a process, or None if it vanished."""
    try:
        s = Path(f"/proc/{pid}/stat").read_text()
    except (FileNotFoundError, ProcessLookupError, PermissionError):
        return None
    rest = s[s.rfind(")") + 2:].split()
    try:
        return rest[0], int(rest[1])
    except (IndexError, ValueError):
        return None


def children_of(parent: int):
    out = []
    for e in Path("/proc").iterdir():
        if not e.name.isdecimal():
            continue
        st = _proc_stat(int(e.name))
        if st and st[1] == parent:
            out.append((int(e.name), st[0]))
    return out


def descendants(root: int) -> list[int]:
    """All live descendants of ``root`` (breadth first), excluding root."""
    parent_of = {}
    for e in Path("/proc").iterdir():
        if e.name.isdecimal():
            st = _proc_stat(int(e.name))
            if st:
                parent_of[int(e.name)] = st[1]
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
    """Reap zombie direct children (adopted orphans) that are not excluded.

    Only zombies are waited for, by pid, so a status owned by a Popen object is
    never consumed by a blanket waitpid(-1)."""
    if not is_subreaper():
        raise RuntimeError("enable_subreaper() must be called before reaping")
    excluded = {int(p) for p in exclude_pids}
    deadline = time.monotonic() + max(0.0, timeout)
    reaped = []
    while True:
        pending = False
        for pid, state in children_of(os.getpid()):
            if pid in excluded:
                continue
            pending = True
            if state != "Z":
                continue
            try:
                done, _ = os.waitpid(pid, os.WNOHANG)
            except ChildProcessError:
                continue
            if done:
                reaped.append(done)
        if not pending or time.monotonic() >= deadline:
            return reaped
        time.sleep(min(0.02, max(0.0, deadline - time.monotonic())))
