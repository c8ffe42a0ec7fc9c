"""Evidence reports from session event logs: recovery-stage timings,
endurance and ABBA throughput, with plots.

    python -m shift_b200.analysis.report --stages SESSION_DIR --output OUT
    python -m shift_b200.analysis.report --endurance SESSION_DIR --output OUT
    python -m shift_b200.analysis.report --bench-flat A1 A2 --bench-shift B1 B2 --output OUT

The reference splits these over shift_full/paper_metrics.py (per-stage
distributions of a recovery: snapshot export, transport send / receive,
state load, audit, process-group reconfiguration; :110-143) and
shift_full/reporting.py (endurance summary :206, ABBA benchmark of flat
against fault-tolerant sessions :330-516, plots :518-610).  Here one module
reads the same JSONL rows (``events_g<G>_r<R>.jsonl`` plus the
``controller_r*.jsonl`` / ``supervisor_r*.jsonl`` logs) and writes JSON, a CSV
of the per-step series and SVG plots drawn directly (no plotting library).
Missing values are omitted, never invented; a session with a failure row or
without commits is never reported complete.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import statistics
from collections import defaultdict
from pathlib import Path

from .trajectory import read_events

FAILURE_KINDS = {"failed", "failure", "unexpected_exit", "supervisor_error", "runtime_error", "worker_failed"}


def _num(v) -> bool:
    return isinstance(v, (int, float)) and not isinstance(v, bool) and math.isfinite(float(v))


def describe(xs) -> dict | None:
    xs = sorted(float(x) for x in xs if _num(x))
    if not xs:
        return None

    def q(f):
        i = f * (len(xs) - 1)
        lo, hi = math.floor(i), math.ceil(i)
        return xs[lo] + (xs[hi] - xs[lo]) * (i - lo)

    return {"n": len(xs), "min": xs[0], "median": q(0.5), "p90": q(0.9), "max": xs[-1],
            "mean": statistics.fmean(xs)}


def _side_logs(session_dir) -> list[dict]:
    rows = []
    for pat in ("controller_r*.jsonl", "supervisor_r*.jsonl", "controller.jsonl"):
        for p in sorted(Path(session_dir).rglob(pat)):
            for line in p.read_text(encoding="utf-8", errors="replace").splitlines():
                try:
                    v = json.loads(line)
                except ValueError:
                    continue
                if isinstance(v, dict):
                    rows.append(v)
    return rows


# --------------------------------------------------------------------------- recovery stages
def stage_distributions(rows) -> dict:
    by = defaultdict(lambda: defaultdict(list))
    begins, ends = defaultdict(list), defaultdict(list)
    for r in rows:
        key = f"rid{r.get('rid')}/rank{r.get('rank')}"
        k = r.get("kind")
        if k == "transport_send":
            by["transport_send_seconds"][key].append(r.get("seconds"))
        elif k == "transport_recv":
            by["transport_recv_seconds"][key].append(r.get("seconds"))
        elif k == "state_loaded":
            by["state_load_seconds"][key].append(r.get("load_seconds"))
        elif k == "restored":
            by["audit_seconds"][key].append(r.get("audit_seconds"))
        elif k == "reconfigure_end":
            by["reconfigure_seconds"][key].append(r.get("seconds"))
        elif k in ("snapshot_begin", "snapshot") and r.get("step") is not None:
            (begins if k == "snapshot_begin" else ends)[(r.get("rid"), r.get("generation"), r.get("rank"),
                                                         r.get("step"))].append(r.get("monotonic"))
    export = []
    for key, starts in begins.items():
        s = sorted(x for x in starts if _num(x))
        e = sorted(x for x in ends.get(key, []) if _num(x))
        export.extend(b - a for a, b in zip(s, e) if b >= a)
    out = {"snapshot_export_seconds": describe(export)}
    for name, per in sorted(by.items()):
        out[name] = {"all": describe([x for xs in per.values() for x in xs]),
                     "by_rank": {k: describe(v) for k, v in sorted(per.items())}}
    return out


# --------------------------------------------------------------------------- endurance
def _commits(rows, rank=0):
    """rank-`rank` commit rows per replica, ordered by time."""
    per = defaultdict(list)
    for r in rows:
        if r.get("kind") == "commit" and r.get("rank", 0) == rank and _num(r.get("time")):
            per[r.get("rid", 0)].append(r)
    for v in per.values():
        v.sort(key=lambda r: r["time"])
    return per


def endurance_summary(session_dir) -> dict:
    rows, errors, nfiles = read_events(session_dir)
    side = _side_logs(session_dir)
    failures = [r for r in rows + side if r.get("kind") in FAILURE_KINDS]
    commits = _commits(rows)
    replicas = {}
    for rid, cs in sorted(commits.items(), key=lambda kv: str(kv[0])):
        times = [c["time"] for c in cs]
        losses = [c.get("loss") for c in cs if _num(c.get("loss"))]
        replicas[str(rid)] = {
            "commits": len(cs), "last_step": max((c.get("step", 0) for c in cs), default=0),
            "commit_interval_seconds": describe([b - a for a, b in zip(times, times[1:])]),
            "loss_first": losses[0] if losses else None, "loss_last": losses[-1] if losses else None,
            "nonfinite_gradients": sum(1 for c in cs if c.get("finite_gradients") is False),
            "generations": sorted({c.get("generation", 0) for c in cs}),
        }
    faults = [r for r in side if r.get("kind") in ("injected", "fault_injected", "fault_recovered")]
    return {"complete": bool(commits) and not failures and not errors, "event_files": nfiles,
            "parse_errors": errors[:10], "failures": [r.get("kind") for r in failures][:20],
            "fault_rows": len(faults), "replicas": replicas, "stages": stage_distributions(rows)}


# --------------------------------------------------------------------------- ABBA bench
def bench_session(session_dir, label, warmup_commits=10, tokens_per_sample=None) -> dict:
    """Steady-state throughput of one session from its rank-0 commits after
    the first `warmup_commits` of each replica."""
    rows, errors, _ = read_events(session_dir)
    ready = [r for r in rows if r.get("kind") == "ready"]
    commits = _commits(rows)
    steps_s, samples = [], []
    for cs in commits.values():
        kept = cs[warmup_commits:]
        times = [c["time"] for c in kept]
        steps_s.extend(b - a for a, b in zip(times, times[1:]))
        samples.extend(len(c.get("sample_ids") or []) for c in kept[1:])
    step = describe(steps_s)
    per_step_samples = statistics.median(samples) if samples else None
    # every replica's commit covers its own samples; the global batch is their sum
    global_samples = per_step_samples * max(1, len(commits)) if per_step_samples else None
    out = {"label": label, "dir": str(session_dir), "replicas": len(commits), "ready_rows": len(ready),
           "step_seconds": step, "samples_per_step": global_samples, "parse_errors": errors[:5]}
    if step and global_samples:
        out["samples_per_second"] = global_samples / step["median"]
        if tokens_per_sample:
            out["tokens_per_second"] = out["samples_per_second"] * tokens_per_sample
    return out


def benchmark_summary(flat_dirs, shift_dirs, warmup_commits=10, tokens_per_sample=None) -> dict:
    """ABBA: flat (A) and fault-tolerant (B) sessions interleaved in time;
    the ratio of medians over the A and B sessions."""
    a = [bench_session(d, f"flat{i}", warmup_commits, tokens_per_sample) for i, d in enumerate(flat_dirs)]
    b = [bench_session(d, f"shift{i}", warmup_commits, tokens_per_sample) for i, d in enumerate(shift_dirs)]

    def med(xs, key):
        vs = [x[key] for x in xs if _num(x.get(key))]
        return statistics.median(vs) if vs else None

    fa, fb = med(a, "samples_per_second"), med(b, "samples_per_second")
    return {"flat": a, "shift": b, "flat_samples_per_second": fa, "shift_samples_per_second": fb,
            "shift_vs_flat_percent": (100.0 * (fb - fa) / fa) if fa and fb else None,
            "complete": bool(a) and bool(b) and fa is not None and fb is not None}


# --------------------------------------------------------------------------- plots
def svg_lines(series: dict, title: str, xlabel: str, ylabel: str, path, width=720, height=360) -> bool:
    """Write an SVG line plot of {name: [(x, y), ...]}; False when no data."""
    pts = [(x, y) for s in series.values() for x, y in s if _num(x) and _num(y)]
    if not pts:
        return False
    x0, x1 = min(p[0] for p in pts), max(p[0] for p in pts)
    y0, y1 = min(p[1] for p in pts), max(p[1] for p in pts)
    x1 = x1 if x1 > x0 else x0 + 1
    y1 = y1 if y1 > y0 else y0 + 1
    L, R, T, B = 70, 20, 40, 50
    sx = lambda x: L + (x - x0) / (x1 - x0) * (width - L - R)   # noqa: E731
    sy = lambda y: height - B - (y - y0) / (y1 - y0) * (height - T - B)   # noqa: E731
    colors = ["#1f77b4", "#d62728", "#2ca02c", "#9467bd", "#ff7f0e", "#17becf"]
    out = [f'<svg xmlns="http://www.w3.org/2000/svg" width="{width}" height="{height}" font-family="sans-serif" '
           f'font-size="12">', f'<rect width="{width}" height="{height}" fill="white"/>',
           f'<text x="{width / 2}" y="20" text-anchor="middle" font-size="14">{title}</text>',
           f'<line x1="{L}" y1="{height - B}" x2="{width - R}" y2="{height - B}" stroke="black"/>',
           f'<line x1="{L}" y1="{T}" x2="{L}" y2="{height - B}" stroke="black"/>',
           f'<text x="{width / 2}" y="{height - 10}" text-anchor="middle">{xlabel}</text>',
           f'<text x="15" y="{height / 2}" text-anchor="middle" transform="rotate(-90 15 {height / 2})">{ylabel}</text>']
    for i in range(5):
        yv = y0 + (y1 - y0) * i / 4
        xv = x0 + (x1 - x0) * i / 4
        out.append(f'<text x="{L - 5}" y="{sy(yv) + 4:.1f}" text-anchor="end">{yv:.4g}</text>')
        out.append(f'<text x="{sx(xv):.1f}" y="{height - B + 16}" text-anchor="middle">{xv:.4g}</text>')
    for n, (name, s) in enumerate(series.items()):
        c = colors[n % len(colors)]
        p = " ".join(f"{sx(x):.1f},{sy(y):.1f}" for x, y in s if _num(x) and _num(y))
        out.append(f'<polyline fill="none" stroke="{c}" stroke-width="1.5" points="{p}"/>')
        out.append(f'<text x="{width - R - 5}" y="{T + 14 * (n + 1)}" text-anchor="end" fill="{c}">{name}</text>')
    out.append("</svg>")
    Path(path).write_text("\n".join(out) + "\n")
    return True


def write_endurance(session_dir, output) -> dict:
    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    summary = endurance_summary(session_dir)
    rows, _, _ = read_events(session_dir)
    commits = _commits(rows)
    with open(output / "endurance_steps.csv", "w", newline="") as f:
        w = csv.writer(f)
        w.writerow(["rid", "step", "time", "loss", "participants", "seconds"])
        for rid, cs in sorted(commits.items(), key=lambda kv: str(kv[0])):
            for c in cs:
                w.writerow([rid, c.get("step"), c.get("time"), c.get("loss"), c.get("participants"), c.get("seconds")])
    t0 = min((c["time"] for cs in commits.values() for c in cs), default=0.0)
    summary["plots"] = {
        "loss": svg_lines({f"replica {rid}": [(c.get("step"), c.get("loss")) for c in cs]
                           for rid, cs in commits.items()}, "loss per committed step", "step", "loss",
                          output / "endurance_loss.svg"),
        "step_time": svg_lines({f"replica {rid}": [(c["time"] - t0, c.get("seconds")) for c in cs]
                                for rid, cs in commits.items()}, "step time", "seconds since first commit",
                               "seconds per step", output / "endurance_step_time.svg"),
    }
    (output / "endurance.json").write_text(json.dumps(summary, indent=1, default=str))
    return summary


def write_bench(flat_dirs, shift_dirs, output, warmup_commits=10, tokens_per_sample=None) -> dict:
    output = Path(output)
    output.mkdir(parents=True, exist_ok=True)
    summary = benchmark_summary(flat_dirs, shift_dirs, warmup_commits, tokens_per_sample)
    series = {}
    for s in summary["flat"] + summary["shift"]:
        if _num(s.get("samples_per_second")):
            series.setdefault(s["label"].rstrip("0123456789"), []).append(
                (len(series.get(s["label"].rstrip("0123456789"), [])), s["samples_per_second"]))
    summary["plots"] = {"bench": svg_lines(series, "ABBA throughput", "session", "samples / s",
                                           output / "bench.svg")}
    (output / "bench.json").write_text(json.dumps(summary, indent=1, default=str))
    return summary


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--stages", default="")
    ap.add_argument("--endurance", default="")
    ap.add_argument("--bench-flat", nargs="*", default=[])
    ap.add_argument("--bench-shift", nargs="*", default=[])
    ap.add_argument("--warmup-commits", type=int, default=10)
    ap.add_argument("--tokens-per-sample", type=int, default=None)
    ap.add_argument("--output", required=True)
    a = ap.parse_args(argv)
    out = Path(a.output)
    out.mkdir(parents=True, exist_ok=True)
    ok = True
    if a.stages:
        rows, _, _ = read_events(a.stages)
        st = stage_distributions(rows)
        (out / "stages.json").write_text(json.dumps(st, indent=1))
        print(json.dumps({"stages": sorted(st)}))
    if a.endurance:
        s = write_endurance(a.endurance, out)
        ok &= s["complete"]
        print(json.dumps({"endurance_complete": s["complete"], "replicas": sorted(s["replicas"])}))
    if a.bench_flat or a.bench_shift:
        s = write_bench(a.bench_flat, a.bench_shift, out, a.warmup_commits, a.tokens_per_sample)
        ok &= s["complete"]
        print(json.dumps({"bench_complete": s["complete"], "shift_vs_flat_percent": s["shift_vs_flat_percent"]}))
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
