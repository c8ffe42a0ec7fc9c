"""Safety pre-flight for GPU sessions, and source provenance checks.

    python -m shift_b200.control.preflight [--gpus 0,1,2] [--provenance results/S/provenance.json]

Two checks the reference runs before a planned-handoff run
(scripts/run_planned_handoff.py:61-65 refuses to start while any GPU compute
process exists; scripts/verify_overlap_source.py:6-17 checks that the sources
in use are the ones recorded):

* ``gpu_idle``: no compute process holds any of the GPUs the session will use
  (read-only ``nvidia-smi --query-compute-apps``; nothing about the GPUs is
  changed).  A measurement or handoff timing taken next to someone else's job
  is not evidence, and a fault test must not share a GPU with another job.
* ``sources_match``: the SHA-256 of every source file of this package equals
  the ``files`` map a supervisor recorded in the session's ``provenance.json``
  (``control/supervisor.py`` writes it at start), so an analysis is known to
  describe the code that ran.

Exit code 0 when every requested check passes.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import subprocess as sp
from pathlib import Path

PKG = Path(__file__).resolve().parents[1]
SOURCE_SUFFIXES = (".py", ".cu", ".cuh", ".cpp", ".hpp", ".h")


def source_hashes(pkg: Path = PKG) -> dict:
    """{path relative to the package's parent: sha256} of every source file
    (the map ``control/supervisor.provenance`` records)."""
    out = {}
    for p in sorted(pkg.rglob("*")):
        if p.is_file() and p.suffix in SOURCE_SUFFIXES and "__pycache__" not in p.parts:
            out[str(p.relative_to(pkg.parent))] = hashlib.sha256(p.read_bytes()).hexdigest()
    return out


def _query(cmd) -> list[str] | None:
    try:
        r = sp.run(cmd, capture_output=True, text=True, timeout=15)
    except (OSError, sp.TimeoutExpired):
        return None
    if r.returncode != 0:
        return None
    return [ln.strip() for ln in r.stdout.splitlines() if ln.strip()]


def gpu_compute_apps(run=_query) -> dict | None:
    """{gpu index: [{"pid", "name", "used_mib"}]} of running compute processes,
    None when nvidia-smi is unavailable."""
    uuids = run(["nvidia-smi", "--query-gpu=index,uuid", "--format=csv,noheader"])
    apps = run(["nvidia-smi", "--query-compute-apps=gpu_uuid,pid,process_name,used_memory",
                "--format=csv,noheader,nounits"])
    if uuids is None or apps is None:
        return None
    index = {}
    for ln in uuids:
        i, _, u = (x.strip() for x in ln.partition(","))
        index[u] = int(i)
    out: dict = {i: [] for i in index.values()}
    for ln in apps:
        parts = [x.strip() for x in ln.split(",")]
        if len(parts) < 4:
            continue
        u, pid, name, mem = parts[:4]
        out.setdefault(index.get(u, -1), []).append(
            {"pid": int(pid) if pid.isdigit() else pid, "name": name, "used_mib": int(mem) if mem.isdigit() else mem})
    return out


def check_gpus_idle(gpus=None, run=_query, ignore_pids=()) -> dict:
    apps = gpu_compute_apps(run)
    if apps is None:
        return {"pass": False, "error": "nvidia-smi unavailable"}
    wanted = sorted(apps) if gpus is None else list(gpus)
    busy = {g: [a for a in apps.get(g, []) if a["pid"] not in set(ignore_pids)] for g in wanted}
    busy = {g: a for g, a in busy.items() if a}
    return {"pass": not busy, "gpus": wanted, "busy": busy}


def check_sources(provenance_path, pkg: Path = PKG) -> dict:
    try:
        rec = json.loads(Path(provenance_path).read_text())["files"]
    except (OSError, ValueError, KeyError) as exc:
        return {"pass": False, "error": f"{type(exc).__name__}: {exc}"}
    now = source_hashes(pkg)
    changed = sorted(k for k in rec.keys() & now.keys() if rec[k] != now[k])
    missing = sorted(rec.keys() - now.keys())
    added = sorted(now.keys() - rec.keys())
    return {"pass": not changed and not missing and not added, "files": len(rec), "changed": changed[:20],
            "missing": missing[:20], "added": added[:20]}


def preflight(gpus=None, provenance=None, run=_query) -> dict:
    checks = {}
    if gpus is not None or provenance is None:
        checks["gpu_idle"] = check_gpus_idle(gpus, run)
    if provenance is not None:
        checks["sources_match"] = check_sources(provenance)
    return {"pass": all(c["pass"] for c in checks.values()), "checks": checks}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", default=None, help="comma-separated GPU indices (default: all)")
    ap.add_argument("--provenance", default=None, help="a session's provenance.json")
    ap.add_argument("--skip-gpus", action="store_true", help="only check the sources")
    a = ap.parse_args(argv)
    gpus = [int(x) for x in a.gpus.split(",")] if a.gpus else None
    checks = {}
    if not a.skip_gpus:
        checks["gpu_idle"] = check_gpus_idle(gpus)
    if a.provenance:
        checks["sources_match"] = check_sources(a.provenance)
    rep = {"pass": bool(checks) and all(c["pass"] for c in checks.values()), "checks": checks}
    print(json.dumps(rep, default=str))
    return 0 if rep["pass"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
