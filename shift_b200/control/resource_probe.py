"""Resource snapshot of a session: GPUs (nvidia-smi) and the session's
processes (/proc RSS and CPU time), like the reference's resource probe
(shift_full/resource_probe.py) but for processes on this host.

    python -m shift_b200.control.resource_probe SESSION_DIR [--append]

Process ids come from the session's ``ready`` / ``launched`` events; the
snapshot is appended to ``<session>/resources.jsonl``.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess as sp
import time
from pathlib import Path

from .event_reader import IncrementalReader

_GPU_FIELDS = "index,memory.used,memory.total,utilization.gpu,power.draw"


def gpus() -> list[dict]:
    try:
        out = sp.run(["nvidia-smi", f"--query-gpu={_GPU_FIELDS}", "--format=csv,noheader,nounits"],
                     capture_output=True, text=True, timeout=10)
    except (OSError, sp.TimeoutExpired):
        return []
    rows = []
    for line in out.stdout.strip().splitlines():
        f = [x.strip() for x in line.split(",")]
        if len(f) == 5:
            rows.append({"index": int(f[0]), "memory_used_mib": float(f[1]), "memory_total_mib": float(f[2]),
                         "utilization_pct": float(f[3]), "power_w": float(f[4]) if f[4] not in ("[N/A]", "") else None})
    return rows


def process(pid: int) -> dict | None:
    try:
        status = Path(f"/proc/{pid}/status").read_text()
        stat = Path(f"/proc/{pid}/stat").read_text().rsplit(")", 1)[1].split()
    except OSError:
        return None
    rss = next((int(line.split()[1]) for line in status.splitlines() if line.startswith("VmRSS:")), 0)
    tick = os.sysconf("SC_CLK_TCK")
    return {"pid": pid, "rss_kib": rss, "cpu_user_s": int(stat[11]) / tick, "cpu_system_s": int(stat[12]) / tick,
            "threads": int(stat[17])}


def snapshot(session_dir) -> dict:
    r = IncrementalReader(session_dir)
    r.poll()
    pids = sorted({x["pid"] for x in r.all_rows if x["kind"] in ("ready", "launched", "supervisor_ready")
                   and isinstance(x.get("pid"), int)})
    procs = [p for p in (process(pid) for pid in pids) if p is not None]
    return {"time": time.time(), "gpus": gpus(), "processes": procs,
            "total_rss_kib": sum(p["rss_kib"] for p in procs)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("session_dir")
    a = ap.parse_args(argv)
    snap = snapshot(a.session_dir)
    with (Path(a.session_dir) / "resources.jsonl").open("a") as f:
        f.write(json.dumps(snap) + "\n")
    print(json.dumps(snap, indent=1))


if __name__ == "__main__":
    main()
