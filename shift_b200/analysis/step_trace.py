"""Per-rank breakdown of one training step from ``bench.py --trace`` timelines.

    python -m shift_b200.analysis.step_trace TRACE_DIR [--out breakdown.json]

Reads every ``trace_n<N>_r<R>.json[.gz]`` (torch profiler chrome traces of one
untimed step per rank) and reports, per rank: the step span on the device
(first kernel start to last kernel end), busy time per kernel category --
GEMMs, attention, MoE routing / permutation, norms / RoPE, the cross-replica
reduction + AdamW (K1), tensor- and pipeline-parallel exchanges and their
waits, the loss, other -- and the idle time on the busiest stream (gaps
between its kernels).  Kernel names are this framework's (namespaces
``sb::gemm``, ``sb::fa``, ``sb::moe``, ``sb::norm``, ``sb::coll``, ...).
"""
from __future__ import annotations

import argparse
import collections
import gzip
import json
import re
from pathlib import Path

CATEGORIES = [
    ("flag_wait", re.compile(r"flag_wait")),
    ("k1_reduce_adamw", re.compile(r"fused_reduce_adamw|reduce_slice_scatter|adamw")),
    ("exchange_copy", re.compile(r"xcopy|peer_copy|flag_set")),
    ("nccl", re.compile(r"nccl", re.I)),
    ("attention", re.compile(r"::fa::|attention")),
    ("gemm", re.compile(r"::gemm::|gemm_kernel|cutlass|sm100_xmma|nvjet", re.I)),
    ("moe", re.compile(r"::moe::")),
    ("norm_rope", re.compile(r"::norm::|rope")),
    ("loss", re.compile(r"xent")),
    ("memset_memcpy", re.compile(r"Memset|Memcpy|FillFunctor|copy_kernel")),
]


def category(name: str) -> str:
    for cat, rx in CATEGORIES:
        if rx.search(name):
            return cat
    return "other"


def load(path: Path) -> list:
    opener = gzip.open if path.suffix == ".gz" else open
    with opener(path, "rt") as f:
        d = json.load(f)
    return [e for e in d.get("traceEvents", []) if e.get("ph") == "X"
            and e.get("cat") in ("kernel", "gpu_memcpy", "gpu_memset")]


def breakdown(events: list) -> dict:
    if not events:
        return {"kernels": 0}
    t0 = min(e["ts"] for e in events)
    t1 = max(e["ts"] + e["dur"] for e in events)
    by_stream = collections.defaultdict(list)
    for e in events:
        by_stream[e.get("tid")].append(e)
    cats = collections.Counter()
    for e in events:
        cats[category(e["name"])] += e["dur"]
    streams = {}
    for tid, es in by_stream.items():
        es.sort(key=lambda e: e["ts"])
        busy = sum(e["dur"] for e in es)
        # idle = span of the stream minus the union of its kernels' intervals
        union, cur_s, cur_e = 0.0, None, None
        for e in es:
            s, t = e["ts"], e["ts"] + e["dur"]
            if cur_e is None or s > cur_e:
                if cur_e is not None:
                    union += cur_e - cur_s
                cur_s, cur_e = s, t
            else:
                cur_e = max(cur_e, t)
        union += cur_e - cur_s
        streams[str(tid)] = {"kernels": len(es), "busy_ms": round(busy / 1e3, 3),
                             "span_ms": round((es[-1]["ts"] + es[-1]["dur"] - es[0]["ts"]) / 1e3, 3),
                             "idle_ms": round(((es[-1]["ts"] + es[-1]["dur"] - es[0]["ts"]) - union) / 1e3, 3)}
    main = max(streams.values(), key=lambda v: v["busy_ms"])
    return {"kernels": len(events), "step_span_ms": round((t1 - t0) / 1e3, 3),
            "busy_ms_by_category": {k: round(v / 1e3, 3) for k, v in cats.most_common()},
            "streams": streams, "main_stream_idle_ms": main["idle_ms"]}


def analyze(trace_dir) -> dict:
    out = {}
    for p in sorted(Path(trace_dir).glob("trace_n*_r*.json*")):
        m = re.search(r"trace_n(\d+)_r(\d+)", p.name)
        out[f"rank{m.group(2)}"] = breakdown(load(p))
        out[f"rank{m.group(2)}"]["n_gpus"] = int(m.group(1))
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("trace_dir")
    ap.add_argument("--out", default="")
    a = ap.parse_args(argv)
    res = analyze(a.trace_dir)
    text = json.dumps(res, indent=1)
    if a.out:
        Path(a.out).write_text(text + "\n")
    print(text)
    return 0 if res else 1


if __name__ == "__main__":
    raise SystemExit(main())
