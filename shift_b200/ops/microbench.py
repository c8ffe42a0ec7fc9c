"""Kernel micro-benchmarks at the shapes of the 0.494B MoE training step.

    python -m shift_b200.ops.microbench [--ops gemm,attn,mem,fused] [--iters N]

Each case is timed with CUDA events on the launching stream after warm-up,
with a synchronize on both sides; inputs of the timed cases are larger than
the 126 MB L2 or an L2-sized buffer is rewritten between iterations.  The
achieved rate is reported against MEASURED_PEAKS.json (the driver-measured
copy bandwidth and cuBLAS bf16 throughput of this GPU type), and GEMMs are
also timed against torch.matmul (cuBLAS) on the same operands.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from . import functional as Fn
from . import gemm as G
from . import reference as ref

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"], "src": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "src": "fallback"}


_flush = None


def flush_l2():
    global _flush
    if _flush is None:
        _flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    _flush.zero_()


def timeit(fn, iters=20, warmup=3, flush=True):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    times.sort()
    return times[len(times) // 2]


def bf(*shape, std=1.0):
    return (torch.randn(*shape, device="cuda") * std).to(torch.bfloat16)


def gemm_cases(T=16384):
    H, F, V, E, k = 1024, 672, 32768, 16, 4
    cases = []
    for (name, M, N, K) in [("qkv", T, 1536, H), ("o", T, H, H), ("lm_head", T, V, H)]:
        x, w = bf(M, K), bf(N, K)
        dy = bf(M, N)
        dw = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        flops = 2.0 * M * N * K
        cases.append((f"{name}.fwd {M}x{N}x{K}", flops, lambda x=x, w=w: G.linear_fwd(x, w),
                      lambda x=x, w=w: torch.matmul(x, w.t())))
        cases.append((f"{name}.dgrad", flops, lambda dy=dy, w=w: G.linear_dgrad(dy, w),
                      lambda dy=dy, w=w: torch.matmul(dy, w)))
        cases.append((f"{name}.wgrad", flops, lambda dy=dy, x=x, dw=dw: G.linear_wgrad(dy, x, dw),
                      lambda dy=dy, x=x: torch.matmul(dy.t(), x)))
    # grouped experts: T*k rows spread uniformly over E experts, padded to 128
    per = T * k // E
    counts = [per] * E
    offs_l = [0]
    for c in counts:
        offs_l.append(offs_l[-1] + (c + 127) // 128 * 128)
    offs = torch.tensor(offs_l, dtype=torch.int32, device="cuda")
    R = offs_l[-1]
    x = bf(R, H)
    w1 = bf(E, 2 * F, H, std=0.02)
    w2 = bf(E, H, F, std=0.02)
    act = bf(R, F)
    dy2 = bf(R, H)
    dh = bf(R, 2 * F)
    dw1 = torch.empty(E, 2 * F, H, device="cuda", dtype=torch.bfloat16)
    dw2 = torch.empty(E, H, F, device="cuda", dtype=torch.bfloat16)
    f1 = 2.0 * R * 2 * F * H
    f2 = 2.0 * R * H * F
    cases += [
        (f"experts.w1.fwd+swiglu {R}x{2*F}x{H}", f1, lambda: G.grouped_fwd(x, w1, offs, swiglu=True), None),
        ("experts.w2.fwd", f2, lambda: G.grouped_fwd(act, w2, offs), None),
        ("experts.w2.dgrad", f2, lambda: G.grouped_dgrad(dy2, w2, offs), None),
        ("experts.w2.wgrad", f2, lambda: G.grouped_wgrad(dy2, act, offs, dw2), None),
        ("experts.w1.dgrad", f1, lambda: G.grouped_dgrad(dh, w1, offs), None),
        ("experts.w1.wgrad", f1, lambda: G.grouped_wgrad(dh, x, offs, dw1), None),
    ]
    return cases


_CASE = None       # substring filter on case names (--case)
_WARMUP = 3


def _want(name: str) -> bool:
    return _CASE is None or _CASE in name


def run_gemm(iters):
    pk = peaks()
    rows = []
    for name, flops, ours, lib in gemm_cases():
        if not _want(name):
            continue
        t = timeit(ours, iters, warmup=_WARMUP)
        row = {"case": name, "ms": round(t, 4), "tflops": round(flops / t / 1e9, 1),
               "frac_of_peak": round(flops / t / 1e9 / pk["bf16_tflops"], 3)}
        if lib is not None and _CASE is None:
            tl = timeit(lib, iters)
            row["cublas_ms"] = round(tl, 4)
            row["vs_cublas"] = round(tl / t, 3)
        rows.append(row)
    return rows


def run_attn(iters, B=8, S=2048, Hq=16, Hkv=4, D=64):
    pk = peaks()
    T = B * S
    qkv = bf(T, (Hq + 2 * Hkv) * D)
    scale = 1 / math.sqrt(D)
    o, lse = Fn.attention_fwd(qkv, B, S, Hq, Hkv, D, scale)
    do = bf(T, Hq * D)
    causal_flops = 4.0 * B * Hq * S * S * D / 2
    tf = timeit(lambda: Fn.attention_fwd(qkv, B, S, Hq, Hkv, D, scale), iters, warmup=_WARMUP)
    tb = timeit(lambda: Fn.attention_bwd(qkv, o, lse, do, B, S, Hq, Hkv, D, scale), iters, warmup=_WARMUP)
    rows = [{"case": f"attn.fwd B{B} S{S} {Hq}q/{Hkv}kv d{D}", "ms": round(tf, 4),
             "tflops": round(causal_flops / tf / 1e9, 1), "frac_of_peak": round(causal_flops / tf / 1e9 / pk["bf16_tflops"], 3)},
            {"case": "attn.bwd", "ms": round(tb, 4), "tflops": round(2.5 * causal_flops / tb / 1e9, 1),
             "frac_of_peak": round(2.5 * causal_flops / tb / 1e9 / pk["bf16_tflops"], 3)}]
    # library yardstick on the same shapes: torch SDPA with each backend it has here
    from torch.nn.attention import SDPBackend, sdpa_kernel
    q = qkv[:, :Hq * D].reshape(B, S, Hq, D).transpose(1, 2).contiguous().requires_grad_(True)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].reshape(B, S, Hkv, D).transpose(1, 2).contiguous().requires_grad_(True)
    v = qkv[:, (Hq + Hkv) * D:].reshape(B, S, Hkv, D).transpose(1, 2).contiguous().requires_grad_(True)
    g = do.reshape(B, S, Hq, D).transpose(1, 2).contiguous()
    for name, be in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION),
                     ("efficient", SDPBackend.EFFICIENT_ATTENTION)):
        try:
            with sdpa_kernel([be]):
                f = lambda: torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale,
                                                                             enable_gqa=True)
                out = f()
                lf = timeit(lambda: f().detach(), iters, warmup=_WARMUP)
                lb = timeit(lambda: torch.autograd.grad(out, (q, k, v), g, retain_graph=True), iters,
                            warmup=_WARMUP)
        except Exception as e:  # a backend may not support these shapes / this GPU
            rows.append({"case": f"sdpa.{name}", "unavailable": type(e).__name__ + ": " + str(e)[:120]})
            continue
        rows.append({"case": f"sdpa.{name}.fwd", "ms": round(lf, 4), "tflops": round(causal_flops / lf / 1e9, 1),
                     "ours_vs_lib": round(lf / tf, 3)})
        rows.append({"case": f"sdpa.{name}.bwd", "ms": round(lb, 4),
                     "tflops": round(2.5 * causal_flops / lb / 1e9, 1), "ours_vs_lib": round(lb / tb, 3)})
    return rows


def run_mem(iters, T=16384, H=1024):
    pk = peaks()
    rows = []
    x, d = bf(T, H), bf(T, H)
    w = bf(H)
    y, rstd, h = Fn.rmsnorm_fwd(x, w, 1e-6, d)
    dw = torch.zeros(H, device="cuda")
    t = timeit(lambda: Fn.rmsnorm_fwd(x, w, 1e-6, d), iters)
    nbytes = T * H * 2 * 4
    rows.append({"case": "add_rmsnorm.fwd", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    t = timeit(lambda: Fn.rmsnorm_bwd(y, h, rstd, w, 1e-6, dw, dres=d), iters)
    nbytes = T * H * 2 * 4
    rows.append({"case": "rmsnorm.bwd", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    n = 124_000_000
    master = torch.randn(n, device="cuda")
    m = torch.zeros(n, device="cuda")
    v = torch.zeros(n, device="cuda")
    g = bf(n)
    outs = [torch.empty_like(master) for _ in range(3)]
    pb = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    t = timeit(lambda: Fn.adamw_step(master, m, v, [g], *outs, pb, 1e-4, 0.9, 0.999, 1e-8, 0.01, 3, 1.0), iters)
    nbytes = n * (2 + 12 + 12 + 2)
    rows.append({"case": f"adamw {n}", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    logits = bf(T, 32768)
    labels = torch.randint(0, 32768, (T,), device="cuda", dtype=torch.int32)
    t = timeit(lambda: Fn.xent_fwd_bwd(logits, labels, 1.0 / T), iters)
    nbytes = T * 32768 * 2 * 2
    rows.append({"case": "xent fwd+bwd", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    from .reference import rope_tables
    cos, sin = rope_tables(2048, 64, 1e6, "cuda")
    qkv = bf(T, 24 * 64)
    t = timeit(lambda: Fn.rope_(qkv, cos, sin, 2048, 20, 64), iters)
    nbytes = T * 20 * 64 * 2 * 2
    rows.append({"case": f"rope {T}x20 heads d64", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    return rows


def run_fused(iters):
    """The fused compute+collective kernels on ONE GPU: every 'peer' buffer is
    a second local tensor (the kernels only see addresses), so the numbers
    are the kernels' own DRAM/tensor work; the NVLink share is measured in the
    multi-GPU step timelines."""
    from ..engine import StepBlock
    from ._ext import ext, status_word
    pk = peaks()
    rows = []
    dev = torch.device("cuda")
    st = status_word(dev)
    blk = StepBlock(dev)
    blk.write(1, 1e-4, 0.9, 0.999, 1)
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    flags[0] = 1 << 30                                   # a peer flag that is always set
    # ---- K1 two-phase: reduce-scatter a slice of two replicas' bf16 grads, then AdamW
    n = 62_000_000                                       # one replica-rank's flat state at 2 x TP2 x PP2
    g0, g1 = bf(n), bf(n)
    red0, red1 = torch.empty_like(g0), torch.empty_like(g0)
    master = torch.randn(n, device=dev)
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    outs = [torch.empty_like(master) for _ in range(3)]
    pb = torch.empty(n, device=dev, dtype=torch.bfloat16)
    nf = torch.zeros(1, dtype=torch.int32, device=dev)
    t = timeit(lambda: ext().reduce_slice_scatter([g0.data_ptr(), g1.data_ptr()], [red0.data_ptr(), red1.data_ptr()],
                                                  0, n // 2, [], blk.dev, 0.5, st, 5.0, 0), iters, warmup=_WARMUP)
    nbytes = (n // 2) * 2 * (2 + 2)                     # read 2 sources, write 2 destinations (bf16)
    rows.append({"case": f"K1.reduce_slice_scatter half of {n}", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    t = timeit(lambda: ext().fused_reduce_adamw([red0.data_ptr()], [], blk.dev, master, m, v, *outs, pb, 0.9, 0.999,
                                                1e-8, 0.01, 1.0, nf, st, 5.0, 0), iters, warmup=_WARMUP)
    nbytes = n * (2 + 12 + 12 + 2)
    rows.append({"case": f"K1.fused_reduce_adamw {n}", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    # ---- TP exchange forms at the 2 x TP2 shapes (8192 tokens per replica, hidden 1024)
    T, H = 8192, 1024
    half = T // 2
    x, d1, d2 = bf(half, H), bf(half, H), bf(half, H)
    w = bf(H, std=0.1) + 1
    gA, gA_peer = bf(T, H), bf(T, H)
    xc = [flags[0].data_ptr(), 0, flags[1].data_ptr(), flags[2].data_ptr(), 0, blk.dev.data_ptr(),
          gA_peer[:half].data_ptr()]
    t = timeit(lambda: Fn.rmsnorm_fwd(x, w, 1e-6, d1, delta2=d2, y_out=gA[:half], xchg=xc), iters, warmup=_WARMUP)
    nbytes = half * H * 2 * (3 + 1 + 2)                   # x, d1, d2 in; h, y (local), y (peer) out
    rows.append({"case": f"K2.rmsnorm_fwd+delta2+push {half}x{H}", "ms": round(t, 4),
                 "gbs": round(nbytes / t / 1e6, 1), "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    wq = bf(768, H)
    from . import gemm as Gm
    xq = [flags[0].data_ptr(), 0, 0, 0, 0, blk.dev.data_ptr(), 0]
    t = timeit(lambda: Gm.linear_fwd(gA, wq, xchg=xq, tp=(half, T, 0, 0, 0, 0)), iters, warmup=_WARMUP)
    flops = 2.0 * T * 768 * H
    rows.append({"case": f"K2.qkv GEMM (gathered A, peer wait) {T}x768x{H}", "ms": round(t, 4),
                 "tflops": round(flops / t / 1e9, 1), "frac_of_peak": round(flops / t / 1e9 / pk["bf16_tflops"], 3)})
    o, wo = bf(T, 512), bf(H, 512)
    own, peer = torch.empty(half, H, dtype=torch.bfloat16, device=dev), torch.empty(half, H, dtype=torch.bfloat16,
                                                                                     device=dev)
    xo = [0, 0, flags[3].data_ptr(), flags[4].data_ptr(), 0, blk.dev.data_ptr(), peer.data_ptr()]
    t = timeit(lambda: Gm.linear_fwd(o, wo, out=own, xchg=xo, tp=(0, 0, half // 128, half, T, 0)), iters,
               warmup=_WARMUP)
    flops = 2.0 * T * H * 512
    rows.append({"case": f"K3.o-proj GEMM -> peer rows {T}x{H}x512", "ms": round(t, 4),
                 "tflops": round(flops / t / 1e9, 1), "frac_of_peak": round(flops / t / 1e9 / pk["bf16_tflops"], 3)})
    # ---- K4 combine with peer-row stores (8 local experts of 16, top-4)
    k = 4
    R = T * k // 2
    y = bf(R, H)
    pos = torch.randint(0, R, (T, k), device=dev, dtype=torch.int32)
    pos[torch.rand(T, k, device=dev) < 0.5] = -1
    wts = torch.rand(T, k, device=dev)
    cown = torch.empty(half, H, dtype=torch.bfloat16, device=dev)
    cpeer = torch.empty(half, H, dtype=torch.bfloat16, device=dev)
    xcmb = [0, 0, flags[5].data_ptr(), flags[6].data_ptr(), 0, blk.dev.data_ptr(), cpeer.data_ptr()]
    t = timeit(lambda: Fn.combine(y, pos, wts, T, cown, (half, T, 0), xcmb), iters, warmup=_WARMUP)
    nbytes = R * H * 2 + T * H * 2
    rows.append({"case": f"K4.combine -> peer rows T{T} k{k}", "ms": round(t, 4), "gbs": round(nbytes / t / 1e6, 1),
                 "frac_of_peak": round(nbytes / t / 1e6 / pk["hbm_gbs"], 3)})
    torch.cuda.synchronize()
    assert int(st[0]) == 0, f"status word {int(st[0])}"
    return rows


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--ops", default="gemm,attn,mem")
    p.add_argument("--iters", type=int, default=20)
    p.add_argument("--case", default=None, help="only GEMM cases whose name contains this (no cuBLAS comparison)")
    p.add_argument("--warmup", type=int, default=3)
    args = p.parse_args()
    global _CASE, _WARMUP
    _CASE, _WARMUP = args.case, args.warmup
    torch.manual_seed(0)
    out = {"peaks": peaks()}
    ops = args.ops.split(",")
    if "gemm" in ops:
        out["gemm"] = run_gemm(args.iters)
    if "attn" in ops:
        out["attn"] = run_attn(args.iters)
    if "mem" in ops:
        out["mem"] = run_mem(args.iters)
    if "fused" in ops:
        out["fused"] = run_fused(args.iters)
    for k, v in out.items():
        if isinstance(v, list):
            for r in v:
                print(json.dumps(r))
    print(json.dumps({"peaks": out["peaks"]}))


if __name__ == "__main__":
    main()
