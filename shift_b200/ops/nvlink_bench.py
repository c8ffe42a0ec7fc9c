"""Fused compute + collective kernels on real peer memory (2 GPUs).

    python -m torch.distributed.run --nproc-per-node 2 -m shift_b200.ops.nvlink_bench [--iters 20]

Both ranks run each kernel at the same time with the other GPU as the peer,
as in training (every exchange is symmetric), so each NVLink direction
carries one rank's traffic.  Peer buffers are the other rank's allocations
mapped over CUDA IPC; the flags a kernel waits on are the peer's, preset so
that the wait passes at once (the measurement is the data movement, not the
schedule).  Timed with CUDA events after warm-up, the max over ranks.

For each kernel the roofline time is the slowest of: its FLOPs at the
measured bf16 GEMM peak, its local HBM bytes at the measured copy bandwidth,
and the bytes it moves over NVLink at 770 GB/s per direction (the measured
peer-copy rate of this machine type; 900 GB/s nominal).  Reported: bytes
over NVLink, achieved NVLink GB/s and achieved time / roofline time
("frac_of_roofline", 1.0 = at the roofline).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

from . import functional as Fn
from . import gemm as G
from ._ext import ext, status_word
from .microbench import peaks

NVLINK_GBS = 770.0


def _time(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    ms = torch.tensor([a.elapsed_time(b) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def _row(name, ms, nvlink_bytes, hbm_bytes=0.0, flops=0.0, pk=None):
    t_roof = max(flops / (pk["bf16_tflops"] * 1e9), hbm_bytes / (pk["hbm_gbs"] * 1e6),
                 nvlink_bytes / (NVLINK_GBS * 1e6))
    bound = max((("compute", flops / (pk["bf16_tflops"] * 1e9)), ("hbm", hbm_bytes / (pk["hbm_gbs"] * 1e6)),
                 ("nvlink", nvlink_bytes / (NVLINK_GBS * 1e6))), key=lambda x: x[1])[0]
    return {"case": name, "ms": round(ms, 4), "nvlink_bytes": int(nvlink_bytes),
            "nvlink_gbs": round(nvlink_bytes / ms / 1e6, 1), "roofline_ms": round(t_roof, 4), "bound": bound,
            "frac_of_roofline": round(t_roof / ms, 3)}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    if dist.get_world_size() != 2:
        raise SystemExit("run on exactly 2 GPUs")
    from ..engine import StepBlock
    from ..parallel.symmetric import SymmetricHeap
    pk = peaks()
    store = dist.distributed_c10d._get_default_store()
    heap = SymmetricHeap(store, f"nv{rank}", dev)
    peer = f"nv{1 - rank}"
    torch.manual_seed(rank)
    blk = StepBlock(dev)
    blk.write(1, 1e-4, 0.9, 0.999, 1)
    st = status_word(dev)
    # ---- symmetric buffers
    n = 64 * 1024 * 1024                       # one gradient bucket (elements)
    T, H = 8192, 1024                          # tokens per replica at 2 x TP2 (one microbatch), hidden
    half = T // 2
    grad = heap.alloc("grad", n * 2).view(torch.bfloat16)[:n]
    red = heap.alloc("red", n * 2).view(torch.bfloat16)[:n]
    gA = heap.alloc("gA", T * H * 2).view(torch.bfloat16)[: T * H].view(T, H)
    rcv = heap.alloc("rcv", half * H * 2).view(torch.bfloat16)[: half * H].view(half, H)
    state = heap.alloc("state", 1 << 30).view(torch.uint8)
    flags = heap.alloc("flags", 4096).view(torch.int32)
    flags.zero_()                              # CTA counters (odd slots 2, 4, 6) start at zero
    for i in (0, 1, 3, 5):
        flags[i] = 1 << 30                     # every flag a peer may wait on is already "set"
    grad.copy_(torch.randn(n, device=dev).to(torch.bfloat16))
    dist.barrier()
    p_grad = heap.open(peer, "grad").view(torch.bfloat16)[:n]
    p_red = heap.open(peer, "red").view(torch.bfloat16)[:n]
    p_gA = heap.open(peer, "gA").view(torch.bfloat16)[: T * H].view(T, H)
    p_rcv = heap.open(peer, "rcv").view(torch.bfloat16)[: half * H].view(half, H)
    p_state = heap.open(peer, "state").view(torch.uint8)
    p_flags = heap.open(peer, "flags").view(torch.int32)
    own_rows = slice(rank * half, (rank + 1) * half)
    rows = []
    sd = blk.dev
    # ---- K1 one-phase: both replicas' bf16 bucket summed in fp32 inside AdamW (peer read over NVLink)
    master = torch.randn(n, device=dev)
    m, v = torch.zeros(n, device=dev), torch.zeros(n, device=dev)
    outs = [torch.empty_like(master) for _ in range(3)]
    pb = torch.empty(n, device=dev, dtype=torch.bfloat16)
    nf = torch.zeros(1, dtype=torch.int32, device=dev)
    srcs = [grad.data_ptr(), p_grad.data_ptr()] if rank == 0 else [p_grad.data_ptr(), grad.data_ptr()]
    ms = _time(lambda: ext().fused_reduce_adamw(srcs, [p_flags[0].data_ptr()], sd, master, m, v, *outs, pb, 0.9,
                                                0.999, 1e-8, 0.01, 0.5, nf, st, 10.0, 0), a.iters, a.warmup)
    rows.append(_row(f"K1 one-phase reduce+AdamW, bucket {n}", ms, n * 2, n * (2 + 12 + 12 + 2), pk=pk))
    # ---- K1 two-phase, phase A: reduce my half-slice from both, store it into both reduced buffers
    lo, hi = (0, n // 2) if rank == 0 else (n // 2, n)
    ms = _time(lambda: ext().reduce_slice_scatter(srcs, [red.data_ptr(), p_red.data_ptr()], lo, hi,
                                                  [p_flags[0].data_ptr()], sd, 0.5, st, 10.0, 0), a.iters, a.warmup)
    rows.append(_row(f"K1 two-phase A (reduce-scatter + all-gather), bucket {n}", ms, (n // 2) * 2 * 2,
                     (n // 2) * 2 * 2, pk=pk))
    # ---- K2: RMSNorm writes this rank's rows into both gather buffers (peer rows over NVLink)
    x, d1, d2 = [torch.randn(half, H, device=dev).to(torch.bfloat16) for _ in range(3)]
    w = (torch.randn(H, device=dev) * 0.1 + 1).to(torch.bfloat16)
    xc = [p_flags[0].data_ptr(), 0, flags[1].data_ptr(), flags[2].data_ptr(), 0, sd.data_ptr(),
          p_gA[own_rows].data_ptr()]
    ms = _time(lambda: Fn.rmsnorm_fwd(x, w, 1e-6, d1, delta2=d2, y_out=gA[own_rows], xchg=xc), a.iters, a.warmup)
    rows.append(_row(f"K2 RMSNorm + push own rows to the peer {half}x{H}", ms, half * H * 2, half * H * 2 * 5, pk=pk))
    # ---- K2: the gathered column-parallel GEMM (peer rows already in local HBM; waits on the peer flag)
    wq = (torch.randn(768, H, device=dev) * 0.02).to(torch.bfloat16)
    plo, phi = (half, T) if rank == 0 else (0, half)
    xq = [p_flags[1].data_ptr(), 0, 0, 0, 0, sd.data_ptr(), 0]
    ms = _time(lambda: G.linear_fwd(gA, wq, xchg=xq, tp=(plo, phi, (rank * half) // 128, 0, 0, 0)), a.iters,
               a.warmup)
    rows.append(_row(f"K2 QKV GEMM on the gathered rows {T}x768x{H}", ms, 0, (T * H + 768 * H + T * 768) * 2,
                     2.0 * T * 768 * H, pk=pk))
    # ---- K3: row-parallel GEMM whose peer-owned output tiles go straight into the peer's buffer
    o = torch.randn(T, 512, device=dev).to(torch.bfloat16)
    wo = (torch.randn(H, 512, device=dev) * 0.02).to(torch.bfloat16)
    own_out = torch.empty(half, H, dtype=torch.bfloat16, device=dev)
    xo = [0, 0, flags[3].data_ptr(), flags[4].data_ptr(), 0, sd.data_ptr(), p_rcv.data_ptr()]
    ms = _time(lambda: G.linear_fwd(o, wo, out=own_out, xchg=xo, tp=(0, 0, ((1 - rank) * half) // 128, plo, phi,
                                                                       own_rows.start)), a.iters, a.warmup)
    rows.append(_row(f"K3 o-proj GEMM, peer rows -> peer {T}x{H}x512", ms, half * H * 2,
                     (T * 512 + H * 512 + half * H) * 2, 2.0 * T * H * 512, pk=pk))
    # ---- K4: MoE combine, the peer's rows stored into the peer's receive buffer
    k = 4
    R = T * k // 2
    y = torch.randn(R, H, device=dev).to(torch.bfloat16)
    pos = torch.randint(0, R, (T, k), device=dev, dtype=torch.int32)
    pos[torch.rand(T, k, device=dev) < 0.5] = -1
    wts = torch.rand(T, k, device=dev)
    cown = torch.empty(half, H, dtype=torch.bfloat16, device=dev)
    xcmb = [0, 0, flags[5].data_ptr(), flags[6].data_ptr(), 0, sd.data_ptr(), p_rcv.data_ptr()]
    ms = _time(lambda: Fn.combine(y, pos, wts, T, cown, (plo, phi, own_rows.start), xcmb), a.iters, a.warmup)
    rows.append(_row(f"K4 MoE combine, peer rows -> peer T{T} top{k}", ms, half * H * 2, (R * H + T * H) * 2, pk=pk))
    # ---- K10: live-state mover, 1 GiB pulled from the peer's HBM
    dst = torch.empty(1 << 30, dtype=torch.uint8, device=dev)
    ms = _time(lambda: ext().peer_copy(p_state.data_ptr(), dst.data_ptr(), 1 << 30), a.iters, a.warmup)
    rows.append(_row("K10 state mover: 1 GiB peer HBM -> local", ms, 1 << 30, 1 << 30, pk=pk))
    torch.cuda.synchronize()
    status = int(st[0])
    dist.barrier()
    heap.close_peers()
    if rank == 0:
        for r in rows:
            print(json.dumps(r))
        print(json.dumps({"peaks": pk, "nvlink_gbs_per_direction": NVLINK_GBS, "status_word": status}))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
