"""ABBA throughput comparison of flat and fault-tolerant training.

    python -m shift_b200.control.abba --gpus 2 [--rounds 2] [--steps 20] [--warmup 5] [--out FILE]

Runs the headline benchmark (``bench.py``, one process per GPU under
``torch.distributed.run``) in the order A B B A per round, so slow drift of
the machine (clocks, temperature, neighbours) hits both arms alike -- the
design of the reference's interleaved flat / SHIFT sessions
(scripts/run_v1_experiments.py:101-110; result RESULTS.md:20).

* A, flat: no fault-tolerance control plane (``SHIFT_BENCH_FT=0``): no
  lighthouse quorum and no commit vote per step.
* B, fault-tolerant: every step takes a quorum of all replicas and commits
  only after the replicas' vote (``SHIFT_BENCH_FT=1``).

Both arms run the same layout and kernels, so the difference is the cost of
fault tolerance.  Each run's device-timed tokens/s (max over ranks) is
parsed from its JSON line; the summary gives per-arm medians and the
throughput change of B against A in percent.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess as sp
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]


def bench_command(gpus: int, steps: int, warmup: int, port: int) -> list:
    base = [sys.executable, str(ROOT / "bench.py"), "--gpus", str(gpus), "--steps", str(steps), "--warmup",
            str(warmup), "--no-check", "--no-k1-compare", "--no-launch-count"]
    if gpus == 1:
        return base
    return [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={gpus}",
            "--master-addr", "127.0.0.1", "--master-port", str(port)] + base[1:]


def parse_line(text: str) -> dict | None:
    for line in reversed(text.splitlines()):
        line = line.strip()
        if line.startswith("{") and '"metric"' in line:
            try:
                return json.loads(line)
            except ValueError:
                return None
    return None


ARMS = {"A": ("flat", {"SHIFT_BENCH_FT": "0"}), "B": ("fault_tolerant", {"SHIFT_BENCH_FT": "1"})}


def run_abba(gpus: int, rounds: int, steps: int, warmup: int, command=bench_command, timeout: float = 900.0,
             port0: int = 29640, log_dir: Path | None = None) -> dict:
    runs = []
    order = "ABBA" * rounds
    for i, arm in enumerate(order):
        name, env_delta = ARMS[arm]
        env = dict(os.environ)
        env.update(env_delta)
        cmd = command(gpus, steps, warmup, port0 + i)
        t0 = time.time()
        p = sp.run(cmd, env=env, capture_output=True, text=True, timeout=timeout, cwd=str(ROOT))
        line = parse_line(p.stdout)
        if log_dir is not None:
            log_dir.mkdir(parents=True, exist_ok=True)
            (log_dir / f"abba_{i:02d}_{arm}.log").write_text(p.stdout + "\n---- stderr ----\n" + p.stderr[-20000:])
        runs.append({"index": i, "arm": arm, "label": name, "returncode": p.returncode, "wall_s": time.time() - t0,
                     "tokens_per_s": line.get("value") if line else None,
                     "ms_per_step": line.get("ms_per_step") if line else None,
                     "clocks": line.get("clocks") if line else None})
    return summarize(runs, gpus, steps, warmup)


def summarize(runs: list, gpus: int, steps: int, warmup: int) -> dict:
    def med(arm):
        xs = [r["tokens_per_s"] for r in runs if r["arm"] == arm and r["tokens_per_s"]]
        return statistics.median(xs) if xs else None

    a, b = med("A"), med("B")
    return {"gpus": gpus, "steps": steps, "warmup": warmup, "order": "".join(r["arm"] for r in runs), "runs": runs,
            "flat_tokens_per_s": a, "fault_tolerant_tokens_per_s": b,
            "fault_tolerant_vs_flat_percent": (100.0 * (b - a) / a) if a and b else None,
            "complete": all(r["returncode"] == 0 and r["tokens_per_s"] for r in runs)}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=2)
    ap.add_argument("--rounds", type=int, default=2)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--out", default="")
    ap.add_argument("--logs", default="")
    a = ap.parse_args(argv)
    res = run_abba(a.gpus, a.rounds, a.steps, a.warmup, log_dir=Path(a.logs) if a.logs else None)
    text = json.dumps(res, indent=1)
    if a.out:
        Path(a.out).parent.mkdir(parents=True, exist_ok=True)
        Path(a.out).write_text(text + "\n")
    print(text)
    return 0 if res["complete"] else 1


if __name__ == "__main__":
    raise SystemExit(main())
