"""Replica launcher: start ``nproc`` ranks of one replica and wait for them.

    python -m shift_b200.control.launch --nproc 4 --master-port P \
        [--devices 0,1,2,3] --module shift_b200.ft.train -- <trainer args>

Each rank gets RANK / LOCAL_RANK / WORLD_SIZE / LOCAL_WORLD_SIZE /
MASTER_ADDR=127.0.0.1 / MASTER_PORT and, with ``--devices``,
SHIFT_CUDA_DEVICE.  The launcher exits with the first non-zero rank status
after terminating the other ranks, like torchrun's behaviour under
``--max_restarts=0`` that the reference relies on (shift_full/supervisor.py:203-248).
It is a light native replacement for torchrun (no rendezvous agent), which is
what keeps the relaunch of a killed replica short.

``--fork``: the ranks are forked from this process and run the trainer
module in-process (``runpy``) instead of exec'ing a new interpreter.  A
supervisor that has already imported torch and the trainer (without touching
CUDA) forks the launcher the same way, so a relaunched replica starts with
every module loaded -- the reference's fork preload
(shift_full/fast_launch.py:27-97, shift_full/launch_server.py).
"""
from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import time


class ForkedProcess:
    """The part of ``subprocess.Popen`` the launchers use, for a forked child."""

    def __init__(self, pid: int):
        self.pid = pid
        self.returncode = None

    @classmethod
    def start(cls, body, log_path=None, new_session=False) -> "ForkedProcess":
        sys.stdout.flush()
        sys.stderr.flush()
        pid = os.fork()
        if pid == 0:                                  # child
            code = 1
            try:
                if new_session:
                    os.setsid()
                if log_path is not None:
                    fd = os.open(log_path, os.O_WRONLY | os.O_CREAT | os.O_APPEND, 0o644)
                    os.dup2(fd, 1)
                    os.dup2(fd, 2)
                    os.close(fd)
                code = body() or 0
            except SystemExit as e:
                code = e.code if isinstance(e.code, int) else (0 if e.code is None else 1)
            except BaseException:
                import traceback
                traceback.print_exc()
                code = 1
            finally:
                try:
                    sys.stdout.flush()
                    sys.stderr.flush()
                finally:
                    os._exit(code)
        return cls(pid)

    def poll(self):
        if self.returncode is None:
            try:
                got, status = os.waitpid(self.pid, os.WNOHANG)
            except ChildProcessError:                 # collected elsewhere (e.g. an orphan reaper)
                self.returncode = -signal.SIGKILL
                return self.returncode
            if got == self.pid:
                self.returncode = os.waitstatus_to_exitcode(status)
        return self.returncode

    def wait(self, timeout=None):
        end = None if timeout is None else time.monotonic() + timeout
        while self.poll() is None:
            if end is not None and time.monotonic() > end:
                raise subprocess.TimeoutExpired(f"pid {self.pid}", timeout)
            time.sleep(0.01)
        return self.returncode

    def send_signal(self, sig):
        if self.poll() is None:
            os.kill(self.pid, sig)

    def terminate(self):
        self.send_signal(signal.SIGTERM)

    def kill(self):
        self.send_signal(signal.SIGKILL)


def run_module_in_child(module: str, args: list, env: dict):
    """Body of a forked rank: its environment, then the module as __main__."""
    import runpy
    os.environ.clear()
    os.environ.update(env)
    sys.argv = [module, *args]
    runpy.run_module(module, run_name="__main__", alter_sys=True)
    return 0


def usable_port(host: str, port: int) -> int:
    """``port`` if it can be bound on ``host`` now, else one the OS picks.
    The launcher is the parent of every local rank, so it can settle the
    rendezvous and manager-store ports for all of them: a configured port can
    already be held by another process's outgoing connection (EADDRINUSE)."""
    import socket
    with socket.socket() as s:
        try:
            s.bind((host, port))
            return port
        except OSError:
            s.bind((host, 0))
            return s.getsockname()[1]


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--nproc", type=int, default=1)
    p.add_argument("--master-addr", default="127.0.0.1")
    p.add_argument("--master-port", type=int, default=29600)
    p.add_argument("--devices", default="")
    p.add_argument("--module", required=True)
    p.add_argument("--fork", action="store_true", help="fork the ranks from this (preloaded) process")
    p.add_argument("rest", nargs=argparse.REMAINDER)
    a = p.parse_args(argv)
    rest = a.rest[1:] if a.rest and a.rest[0] == "--" else a.rest
    devices = [d for d in a.devices.split(",") if d] if a.devices else []
    a.master_port = usable_port(a.master_addr, a.master_port)
    store = os.environ.get("SHIFT_STORE_PORT")
    if store and int(store) > 0:
        os.environ["SHIFT_STORE_PORT"] = str(usable_port(a.master_addr, int(store)))
    procs = []
    for r in range(a.nproc):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(a.nproc),
                   LOCAL_WORLD_SIZE=str(a.nproc), MASTER_ADDR=a.master_addr, MASTER_PORT=str(a.master_port))
        if devices:
            env["SHIFT_CUDA_DEVICE"] = devices[r % len(devices)]
        if a.fork:
            procs.append(ForkedProcess.start(lambda env=env: run_module_in_child(a.module, rest, env)))
        else:
            procs.append(subprocess.Popen([sys.executable, "-m", a.module, *rest], env=env))

    def forward(sig, _frame):
        for q in procs:
            if q.poll() is None:
                try:
                    q.send_signal(sig)
                except ProcessLookupError:
                    pass

    signal.signal(signal.SIGTERM, forward)
    signal.signal(signal.SIGINT, forward)
    code = 0
    while True:
        alive = [q for q in procs if q.poll() is None]
        failed = [q for q in procs if q.poll() not in (None, 0)]
        if failed:
            code = failed[0].returncode
            for q in alive:
                q.terminate()
            deadline = time.monotonic() + 5
            for q in alive:
                try:
                    q.wait(max(0.1, deadline - time.monotonic()))
                except subprocess.TimeoutExpired:
                    q.kill()
            break
        if not alive:
            break
        time.sleep(0.05)
    sys.exit(code if code >= 0 else 128 - code)


if __name__ == "__main__":
    main()
