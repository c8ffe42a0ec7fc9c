"""GEMM entry points on the sm_100a tcgen05 kernel (``csrc/gemm_sm100.cu``).

Naming follows the training step of a linear layer ``y = x @ w.T``:

* ``linear_fwd``   y[M,N]  = x[M,K] @ w[N,K]^T        (A K-major, B K-major)
* ``linear_dgrad`` dx[M,K] = dy[M,N] @ w[N,K]         (A K-major, B MN-major)
* ``linear_wgrad`` dw[N,K] (+)= dy[M,N]^T @ x[M,K]    (A MN-major, B MN-major)

and the grouped (MoE expert) forms, where rows of ``x`` are split into
contiguous per-expert segments by ``offs`` (int32 [G+1], device):

* ``grouped_fwd``   y[r]  = x[r] @ w[g]^T        w [G, N, K]
* ``grouped_dgrad`` dx[r] = dy[r] @ w[g]         w [G, N, K]
* ``grouped_wgrad`` dw[g] (+)= dy[seg g]^T @ x[seg g]

CPU tensors fall back to fp32 ``torch.matmul`` (oracle / CPU harness only).
"""
from __future__ import annotations

import torch

from ._ext import ext, status_word

ROW_GROUPS, K_GROUPS = 0, 1
EPI_BF16, EPI_F32, EPI_ACC_BF16, EPI_ACC_F32, EPI_SWIGLU, EPI_SWIGLU_BWD = 0, 1, 2, 3, 4, 5


_SMS = 148
# relative mainloop efficiency of a tile width (shared-memory operand traffic
# per MMA flop grows as tiles narrow)
_BN_COST = {256: 1.0, 192: 0.95, 128: 0.7}     # measured: 128-wide tiles lose ~25 % at K = 1024


def pick_bn(n: int, tiles_m: int | None = None, sms: int = _SMS) -> int:
    """Tile width maximising (useful columns / padded columns) x (full waves
    / started waves of the persistent grid) x the width's own efficiency.
    Without the row-tile count only the column padding is considered."""
    best, score = 256, -1.0
    for bn in (256, 192, 128):
        tn = -(-n // bn)
        s = n / (tn * bn) * _BN_COST[bn]
        if tiles_m:
            tiles = tiles_m * tn
            waves = tiles / sms
            s *= waves / (-(-tiles // sms))
        if s > score + 1e-9:
            best, score = bn, s
    return best


def pick_bn_split_k(n: int, tiles_m: int, k: int, sms: int = _SMS) -> int:
    """Tile width for a dense weight gradient, which the kernel entry splits
    along K into S = min(sms // tiles, k // 1024) slices when the output has
    few tiles: the width is chosen for the filled fraction of the grid after
    that split (wide tiles split further and keep their higher mainloop
    efficiency, where the padding-only rule above prefers narrow ones)."""
    best, score = 256, -1.0
    for bn in (256, 192, 128):
        tn = -(-n // bn)
        tiles = tiles_m * tn
        split = max(1, min(sms // max(tiles, 1), k // 1024))
        ctas = tiles * split
        fill = ctas / (-(-ctas // sms) * sms)
        s = n / (tn * bn) * _BN_COST[bn] * fill * (0.98 ** (split - 1))   # each slice adds a reduction pass
        if s > score + 1e-9:
            best, score = bn, s
    return best


def _run(A, B, D, D2, offs, M, N, K, G, mode, a_mn, b_mn, epi, alpha, max_rows, xchg=(), tp=()):
    tiles_m = -(-max_rows // 128) if mode == ROW_GROUPS else G * -(-M // 128)
    if mode == ROW_GROUPS and G > 1:
        tiles_m = None                  # grouped: the row split is data dependent
    if mode == K_GROUPS and G == 1 and offs is None and epi != EPI_SWIGLU and not (xchg and xchg[2]):
        bn = pick_bn_split_k(N, tiles_m, K)
    else:
        bn = pick_bn(N, tiles_m)
    if epi == EPI_SWIGLU and bn == 256 and N % 192 == 0:
        bn = 192                        # the SwiGLU activation is staged for TMA stores below 256
    ext().gemm(A, B, D, D2, offs, M, N, K, G, mode, a_mn, b_mn, epi, float(alpha), bn,
               status_word(A.device), max_rows, list(xchg), list(tp))


def _cpu_split(y_full, out, xchg, tp, dtype):
    """CPU stand-in of the kernel's tensor-parallel forms: wait, peer-owned
    output rows to the peer, own rows to ``out``, signal."""
    if xchg and hasattr(xchg, "before"):
        xchg.before()
    if tp and tp[4] > tp[3] and xchg and xchg.peer_out is not None:
        plo, phi, off = tp[3], tp[4], tp[5]
        xchg.peer_out.copy_(y_full[plo:phi])
        keep = torch.ones(y_full.shape[0], dtype=torch.bool)
        keep[plo:phi] = False
        own = y_full[keep]
        del off
    else:
        own = y_full
    res = own.to(dtype) if out is None else out.copy_(own)
    if xchg and hasattr(xchg, "after"):
        xchg.after()
    return res


def linear_fwd(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, xchg=(), tp=()) -> torch.Tensor:
    """``xchg`` / ``tp``: tensor-parallel exchange of the kernel (see
    ``parallel.tp.TPPeer``): a wait on the peer's flag before gathered rows,
    a rotated row-tile order, peer-owned output rows stored into the peer's
    receive buffer (``out`` then holds only this rank's rows) and a signal."""
    M, K = x.shape
    N = w.shape[0]
    if not x.is_cuda:
        if xchg and hasattr(xchg, "before"):
            xchg.before()           # gathered rows must be complete before reading x
            xchg = type(xchg)(None, xchg.sig_ev, xchg.peer_out)
        return _cpu_split(x.float() @ w.float().t(), out, xchg, tp, x.dtype)
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    _run(x, w, out, None, None, M, N, K, 1, ROW_GROUPS, False, False, EPI_BF16, 1.0, M, xchg, tp)
    return out


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, xchg=(), tp=()) -> torch.Tensor:
    M, N = dy.shape
    K = w.shape[1]
    if not dy.is_cuda:
        if xchg and hasattr(xchg, "before"):
            xchg.before()
            xchg = type(xchg)(None, xchg.sig_ev, xchg.peer_out)
        return _cpu_split(dy.float() @ w.float(), out, xchg, tp, dy.dtype)
    if out is None:
        out = torch.empty(M, K, dtype=dy.dtype, device=dy.device)
    _run(dy, w, out, None, None, M, K, N, 1, ROW_GROUPS, False, True, EPI_BF16, 1.0, M, xchg, tp)
    return out


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, dw: torch.Tensor, accumulate: bool = False, xchg=(),
                 tp=()) -> torch.Tensor:
    """dw[N,K] = dy^T x (or +=).  dw may be bf16 or fp32."""
    M, N = dy.shape
    K = x.shape[1]
    if not dy.is_cuda:
        if xchg and hasattr(xchg, "before"):
            xchg.before()
        g = dy.float().t() @ x.float()
        if accumulate:
            dw.add_(g.to(dw.dtype))
        else:
            dw.copy_(g)
        return dw
    if dw.dtype == torch.float32:
        epi = EPI_ACC_F32 if accumulate else EPI_F32
    else:
        epi = EPI_ACC_BF16 if accumulate else EPI_BF16
    _run(dy, x, dw, None, None, N, K, M, 1, K_GROUPS, True, True, epi, 1.0, N, xchg, tp)
    return dw


def grouped_fwd(x: torch.Tensor, w: torch.Tensor, offs: torch.Tensor, swiglu: bool = False):
    """x [R, K] (segments by offs), w [G, N, K].  Returns y [R, N] or, with
    swiglu, (h [R, N], act [R, N/2]) where h holds interleaved gate/up blocks."""
    G, N, K = w.shape
    R = x.shape[0]
    if not x.is_cuda:
        from . import reference as ref
        y = torch.zeros(R, N, dtype=torch.float32)
        o = offs.tolist()
        for g in range(G):
            if o[g + 1] > o[g]:
                y[o[g]:o[g + 1]] = x[o[g]:o[g + 1]].float() @ w[g].float().t()
        y = y.to(x.dtype)
        if swiglu:
            return y, ref.swiglu_interleaved(y)
        return y
    y = torch.empty(R, N, dtype=x.dtype, device=x.device)
    if swiglu:
        act = torch.empty(R, N // 2, dtype=x.dtype, device=x.device)
        _run(x, w.view(G * N, K), y, act, offs, R, N, K, G, ROW_GROUPS, False, False, EPI_SWIGLU, 1.0, R)
        return y, act
    _run(x, w.view(G * N, K), y, None, offs, R, N, K, G, ROW_GROUPS, False, False, EPI_BF16, 1.0, R)
    return y


def grouped_dgrad(dy: torch.Tensor, w: torch.Tensor, offs: torch.Tensor) -> torch.Tensor:
    """dx[r] = dy[r] @ w[g]; dy [R, N], w [G, N, K] -> [R, K]."""
    G, N, K = w.shape
    R = dy.shape[0]
    if not dy.is_cuda:
        out = torch.zeros(R, K, dtype=torch.float32)
        o = offs.tolist()
        for g in range(G):
            if o[g + 1] > o[g]:
                out[o[g]:o[g + 1]] = dy[o[g]:o[g + 1]].float() @ w[g].float()
        return out.to(dy.dtype)
    out = torch.empty(R, K, dtype=dy.dtype, device=dy.device)
    _run(dy, w.view(G * N, K), out, None, offs, R, K, N, G, ROW_GROUPS, False, True, EPI_BF16, 1.0, R)
    return out


def grouped_dgrad_swiglu(dy: torch.Tensor, w: torch.Tensor, offs: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
    """dh = swiglu'(h) applied to dact = dy[r] @ w[g], in the GEMM epilogue:
    dy [R, N], w [G, N, F], h [R, 2F] (interleaved gate/up) -> dh [R, 2F].
    The activation gradient never leaves the chip."""
    G, N, F = w.shape
    R = dy.shape[0]
    if not dy.is_cuda:
        from . import functional as Fn
        return Fn.swiglu_bwd(h, grouped_dgrad(dy, w, offs))
    dh = torch.empty(R, 2 * F, dtype=dy.dtype, device=dy.device)
    _run(dy, w.view(G * N, F), dh, h, offs, R, F, N, G, ROW_GROUPS, False, True, EPI_SWIGLU_BWD, 1.0, R)
    return dh


def grouped_wgrad(dy: torch.Tensor, x: torch.Tensor, offs: torch.Tensor, dw: torch.Tensor,
                  accumulate: bool = False) -> torch.Tensor:
    """dw[g] (+)= dy[seg]^T x[seg]; dy [R, N], x [R, K], dw [G, N, K]."""
    G, N, K = dw.shape
    if not dy.is_cuda:
        o = offs.tolist()
        for g in range(G):
            gr = dy[o[g]:o[g + 1]].float().t() @ x[o[g]:o[g + 1]].float()
            if accumulate:
                dw[g].add_(gr.to(dw.dtype))
            else:
                dw[g].copy_(gr)
        return dw
    if dw.dtype == torch.float32:
        epi = EPI_ACC_F32 if accumulate else EPI_F32
    else:
        epi = EPI_ACC_BF16 if accumulate else EPI_BF16
    _run(dy, x, dw.view(G * N, K), None, offs, N, K, dy.shape[0], G, K_GROUPS, True, True, epi, 1.0, N)
    return dw
