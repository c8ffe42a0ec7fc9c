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
"""
from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import time


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--nproc", type=int, default=1)
    p.add_argument("--master-addr", default="127.0.0.1")
    p.add_argument("--master-port", type=int, default=29600)
    p.add_argument("--devices", default="")
    p.add_argument("--module", required=True)
    p.add_argument("rest", nargs=argparse.REMAINDER)
    a = p.parse_args(argv)
    rest = a.rest[1:] if a.rest and a.rest[0] == "--" else a.rest
    devices = [d for d in a.devices.split(",") if d] if a.devices else []
    procs = []
    for r in range(a.nproc):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE=str(a.nproc),
                   LOCAL_WORLD_SIZE=str(a.nproc), MASTER_ADDR=a.master_addr, MASTER_PORT=str(a.master_port))
        if devices:
            env["SHIFT_CUDA_DEVICE"] = devices[r % len(devices)]
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
