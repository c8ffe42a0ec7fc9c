"""Every sm_100a kernel against a plain fp32 PyTorch statement of the same op."""
import math

import pytest
import torch

from shift_b200.ops import functional as Fn
from shift_b200.ops import gemm as G
from shift_b200.ops import reference as ref
from shift_b200.ops._ext import check_status

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _close(out, expect, tol=2e-2):
    out, expect = out.float(), expect.float()
    scale = expect.abs().max().item() + 1e-6
    err = (out - expect).abs().max().item()
    assert err <= tol * scale, f"max err {err:.4g} vs scale {scale:.4g}"


def _bf(*shape, std=1.0):
    return (torch.randn(*shape, device=DEV) * std).to(torch.bfloat16)


# ----------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (300, 336, 200), (1024, 1536, 1024), (128, 672, 672)])
def test_linear_fwd(M, N, K):
    torch.manual_seed(0)
    x, w = _bf(M, K), _bf(N, K)
    y = G.linear_fwd(x, w)
    torch.cuda.synchronize()
    check_status()
    _close(y, x.float() @ w.float().t())


@pytest.mark.parametrize("M,N,K", [(256, 256, 128), (384, 1024, 672), (200, 512, 1344)])
def test_linear_dgrad(M, N, K):
    torch.manual_seed(1)
    dy, w = _bf(M, N), _bf(N, K)
    dx = G.linear_dgrad(dy, w)
    torch.cuda.synchronize()
    check_status()
    _close(dx, dy.float() @ w.float())


@pytest.mark.parametrize("M", [640, 8192])          # 8192 tokens: split-K path (few output tiles)
@pytest.mark.parametrize("dtype,acc", [(torch.float32, False), (torch.float32, True), (torch.bfloat16, False),
                                       (torch.bfloat16, True)])
def test_linear_wgrad(dtype, acc, M):
    torch.manual_seed(2)
    N, K = 384, 256
    dy, x = _bf(M, N), _bf(M, K)
    base = torch.randn(N, K, device=DEV).to(dtype)
    dw = base.clone()
    G.linear_wgrad(dy, x, dw, accumulate=acc)
    torch.cuda.synchronize()
    check_status()
    expect = dy.float().t() @ x.float() + (base.float() if acc else 0)
    _close(dw, expect)


def _offsets(counts, pad=128):
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + (c + pad - 1) // pad * pad)
    return torch.tensor(offs, dtype=torch.int32, device=DEV)


def _segments(x, counts, offs):
    """zero the padding rows of a [R, C] tensor laid out by offs"""
    o = offs.tolist()
    for g, c in enumerate(counts):
        x[o[g] + c:o[g + 1]] = 0
    return x


# (1344, 1024): the expert w1 shape; (1024, 672): w2, whose data gradient has 672
# columns (a partial last tile, clipped TMA stores)
@pytest.mark.parametrize("N,K", [(1344, 1024), (1024, 672)])
def test_grouped_fwd_dgrad_wgrad(N, K):
    torch.manual_seed(3)
    counts = [130, 0, 5, 256, 77]
    offs = _offsets(counts)
    R = int(offs[-1])
    Gn = len(counts)
    x = _segments(_bf(R, K), counts, offs)
    w = _bf(Gn, N, K, std=0.05)
    y = G.grouped_fwd(x, w, offs)
    dy = _segments(_bf(R, N), counts, offs)
    dx = G.grouped_dgrad(dy, w, offs)
    dw = torch.zeros(Gn, N, K, device=DEV, dtype=torch.bfloat16)
    G.grouped_wgrad(dy, x, offs, dw)
    torch.cuda.synchronize()
    check_status()
    o = offs.tolist()
    for g in range(Gn):
        a, b = o[g], o[g + 1]
        if b > a:
            _close(y[a:b], x[a:b].float() @ w[g].float().t())
            _close(dx[a:b], dy[a:b].float() @ w[g].float())
            _close(dw[g], dy[a:b].float().t() @ x[a:b].float())
        else:
            assert dw[g].abs().max().item() == 0.0


def test_grouped_swiglu_epilogue():
    torch.manual_seed(4)
    counts = [200, 64, 0, 300]
    offs = _offsets(counts)
    R = int(offs[-1])
    Gn, F, K = len(counts), 672, 1024
    x = _bf(R, K)
    w = _bf(Gn, 2 * F, K, std=0.05)
    h, a = G.grouped_fwd(x, w, offs, swiglu=True)
    torch.cuda.synchronize()
    check_status()
    o = offs.tolist()
    for g in range(Gn):
        s, e = o[g], o[g + 1]
        if e > s:
            hr = x[s:e].float() @ w[g].float().t()
            _close(h[s:e], hr)
            _close(a[s:e], ref.swiglu_interleaved(h[s:e].float()))


# ----------------------------------------------------------------------------- norm / rope
@pytest.mark.parametrize("H,res", [(256, True), (1024, True), (1024, False), (512, False)])
def test_rmsnorm_fwd_bwd(H, res):
    torch.manual_seed(5)
    T = 5000
    x, d = _bf(T, H), _bf(T, H)
    w = (1 + 0.1 * torch.randn(H, device=DEV)).to(torch.bfloat16)
    y, rstd, h = Fn.rmsnorm_fwd(x, w, 1e-6, delta=d)
    hr = (x.float() + d.float())
    _close(h, hr)
    _close(y, ref.rmsnorm(h.float(), w.float(), 1e-6))
    dy, dres = _bf(T, H), (_bf(T, H) if res else None)
    dw = torch.zeros(H, device=DEV, dtype=torch.float32)
    dx = Fn.rmsnorm_bwd(dy, h, rstd, w, 1e-6, dw, dres=dres)
    gx, gw = ref.grad_of(lambda a, b: ref.rmsnorm(a, b, 1e-6), [h.float(), w.float()], dy.float())
    _close(dx, gx + dres.float() if res else gx)
    _close(dw, gw, tol=1e-2)
    # deterministic: a second call gives the same bits
    dw2 = torch.zeros_like(dw)
    dx2 = Fn.rmsnorm_bwd(dy, h, rstd, w, 1e-6, dw2, dres=dres)
    assert torch.equal(dx, dx2) and torch.equal(dw, dw2)


@pytest.mark.parametrize("B,S,Hq,Hkv,D,pad", [(2, 128, 4, 2, 64, 0), (3, 101, 16, 4, 64, 0), (2, 64, 8, 2, 128, 0),
                                              (2, 128, 4, 2, 64, 1)])
def test_rope_roundtrip_and_reference(B, S, Hq, Hkv, D, pad):
    """pad = 1: rows of an odd stride (a column view), the unvectorised path."""
    torch.manual_seed(6)
    cos, sin = ref.rope_tables(512, D, 1e6, DEV)
    qkv = _bf(B * S, (Hq + 2 * Hkv) * D + pad)[:, pad:]
    orig = qkv.clone()
    Fn.rope_(qkv, cos, sin, S, Hq + Hkv, D)
    rot = ref.rope(orig[:, : (Hq + Hkv) * D].view(B * S, Hq + Hkv, D).float(), cos, sin, S)
    _close(qkv[:, : (Hq + Hkv) * D].view(B * S, Hq + Hkv, D), rot)
    assert torch.equal(qkv[:, (Hq + Hkv) * D:], orig[:, (Hq + Hkv) * D:])
    Fn.rope_(qkv, cos, sin, S, Hq + Hkv, D, inverse=True)
    _close(qkv, orig)


# ----------------------------------------------------------------------------- attention
# small grids take the head-split dK/dV path, (8, 1024, 16, 4) the direct one
@pytest.mark.parametrize("B,S,Hq,Hkv", [(2, 128, 4, 2), (1, 256, 16, 4), (8, 1024, 16, 4)])
def test_attention_fwd_bwd(B, S, Hq, Hkv):
    torch.manual_seed(7)
    D = 64
    T = B * S
    qkv = _bf(T, (Hq + 2 * Hkv) * D)
    scale = 1 / math.sqrt(D)
    o, lse = Fn.attention_fwd(qkv, B, S, Hq, Hkv, D, scale)

    def f(x):
        q = x[:, : Hq * D].view(T, Hq, D)
        k = x[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
        v = x[:, (Hq + Hkv) * D:].view(T, Hkv, D)
        return ref.attention(q, k, v, B, S, scale).reshape(T, Hq * D)

    _close(o, f(qkv.float()))
    do = _bf(T, Hq * D)
    dqkv = Fn.attention_bwd(qkv, o, lse, do, B, S, Hq, Hkv, D, scale)
    (g,) = ref.grad_of(f, [qkv.float()], do.float())
    _close(dqkv, g, tol=3e-2)


def test_attention_fwd_rescales_when_row_maxima_grow():
    """Keys scaled up along the sequence make later key blocks raise a row's
    maximum by far more than 2^8 (log2 units), so the forward's stale-max
    rescale of O and the row sum runs on many blocks; O and the log-sum-exp
    must still match fp32."""
    torch.manual_seed(11)
    B, S, Hq, Hkv, D = 2, 1024, 4, 2, 64
    T = B * S
    qkv = torch.randn(T, (Hq + 2 * Hkv) * D, device="cuda")
    pos = torch.arange(S, device="cuda").repeat(B).float()
    qkv[:, Hq * D:(Hq + Hkv) * D] *= (1.0 + 12.0 * pos / S)[:, None]
    qkv = qkv.to(torch.bfloat16)
    scale = 1 / math.sqrt(D)
    o, lse = Fn.attention_fwd(qkv, B, S, Hq, Hkv, D, scale)
    x = qkv.float()
    q = x[:, : Hq * D].view(B, S, Hq, D).transpose(1, 2)
    k = x[:, Hq * D:(Hq + Hkv) * D].view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    v = x[:, (Hq + Hkv) * D:].view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(Hq // Hkv, 1)
    sc = (q @ k.transpose(-1, -2)) * scale
    sc = sc.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device="cuda"), 1), float("-inf"))
    ref_lse = torch.logsumexp(sc, -1) / math.log(2.0)                 # base 2, as the kernel stores it
    ref_o = (torch.softmax(sc, -1) @ v).transpose(1, 2).reshape(T, Hq * D)
    # within a row, the later key blocks raise the maximum over the first block by > 8 in log2 units
    growth = (sc.amax(-1) - sc[..., :128].amax(-1)) / math.log(2.0)
    assert float(growth[..., S // 2:].amax()) > 8.0
    _close(o, ref_o)
    assert float((lse - ref_lse).abs().max()) < 2e-2 * float(ref_lse.abs().max())


# ----------------------------------------------------------------------------- MoE plumbing
def test_router_sort_gather_combine():
    torch.manual_seed(8)
    T, H, E, k = 700, 1024, 16, 4
    x = _bf(T, H)
    wr = _bf(E, H, std=0.05)
    probs, idx, w = Fn.router_fwd(x, wr, k, True)
    pr, ir, wref = ref.router(x.float(), wr.float(), k, True)
    _close(probs, pr, tol=1e-3)
    agree = (idx == ir.to(idx.device)).float().mean().item()
    assert agree > 0.99
    pos, offs, counts, row_src = Fn.bucket_sort(idx, 0, E, 128, k)
    # every (token, choice) has a unique slot inside its expert's segment
    o = offs.tolist()
    flat = idx.reshape(-1).tolist()
    pl = pos.tolist()
    assert len(set(pl)) == len(pl)
    for i, (e, p) in enumerate(zip(flat, pl)):
        assert o[e] <= p < o[e] + int(counts[e])
        assert int(row_src[p]) == i // k
    # stability: within an expert, slots follow (token, choice) order
    for e in range(E):
        ps = [p for ee, p in zip(flat, pl) if ee == e]
        assert ps == sorted(ps)
    cap = row_src.shape[0]
    total = offs[E:E + 1]
    xp = Fn.gather_rows(x, row_src, total, cap)
    valid = row_src >= 0
    assert torch.equal(xp[valid], x[row_src[valid].long()])
    y = _bf(cap, H)
    out = Fn.combine(y, pos.view(T, k), w, T)
    expect = torch.zeros(T, H, device=DEV)
    for j in range(k):
        expect += w[:, j:j + 1] * y[pos.view(T, k)[:, j].long()].float()
    _close(out, expect)


def test_router_backward_matches_cpu():
    """dx += d(router)/dx and dWr (sorted top-k weights + auxiliary term) against
    the autograd restatement; T large enough for several token chunks and a
    partial eight-token group in the weight-gradient kernel."""
    torch.manual_seed(12)
    T, H, E, k = 5003, 1024, 16, 4
    x = _bf(T, H)
    wr = _bf(E, H, std=0.05)
    probs, idx, w = Fn.router_fwd(x, wr, k, True)
    dw_topk = torch.randn(T, k, device=DEV)
    aux = torch.randn(E, device=DEV) * 1e-3
    dx = _bf(T, H)
    dx_cpu = dx.cpu().clone()
    dwr = torch.zeros(E, H, device=DEV)
    Fn.router_bwd(x, wr, probs, idx, w, dw_topk, aux, True, dx, dwr)
    dwr_cpu = torch.zeros(E, H)
    Fn.router_bwd(x.cpu(), wr.cpu(), probs.cpu(), idx.cpu(), w.cpu(), dw_topk.cpu(), aux.cpu(), True, dx_cpu,
                  dwr_cpu)
    _close(dx.cpu(), dx_cpu)
    _close(dwr.cpu(), dwr_cpu, tol=1e-2)


def test_bucket_sort_many_chunks_stable():
    """80,000 keys: the per-bin chunk scan runs over several 256-chunk tiles."""
    torch.manual_seed(13)
    n, E, pad = 80_000, 16, 128
    keys = torch.randint(0, E, (n,), device=DEV, dtype=torch.int32)
    keys[::97] = E + 3            # outside [0, E): ignored
    pos, offs, counts, row_src = Fn.bucket_sort(keys, 0, E, pad, 4)
    kc = keys.long().cpu()
    valid = kc < E
    cnt = torch.bincount(kc[valid], minlength=E)
    assert torch.equal(counts.cpu().long(), cnt)
    padded = (cnt + pad - 1) // pad * pad
    o = torch.zeros(E + 1, dtype=torch.long)
    o[1:] = torch.cumsum(padded, 0)
    assert torch.equal(offs.cpu().long(), o)
    # expected slot: bin offset + number of earlier keys of the same bin
    order = torch.argsort(kc.masked_fill(~valid, E), stable=True)
    sk = kc.masked_fill(~valid, E)[order]
    first = torch.searchsorted(sk, torch.arange(E + 1))
    rank_sorted = torch.arange(n) - first[sk]
    expect = torch.full((n,), -1, dtype=torch.long)
    vs = sk < E
    expect[order[vs]] = o[sk[vs]] + rank_sorted[vs]
    assert torch.equal(pos.cpu().long(), expect)
    rs = row_src.cpu().long()
    assert torch.equal(rs[expect[valid]], torch.arange(n)[valid] // 4)


@pytest.mark.parametrize("T,V", [(64, 32768), (700, 32768), (300, 1000), (129, 12288)])
def test_xent_fwd_bwd(T, V):
    torch.manual_seed(9)
    logits = _bf(T, V, std=2.0)
    labels = torch.randint(0, V, (T,), device=DEV, dtype=torch.int32)
    labels[3] = -100
    ref_loss = ref.cross_entropy(logits.float(), labels)
    (g,) = ref.grad_of(lambda z: ref.cross_entropy(z, labels).sum(), [logits.float()], torch.tensor(1.0, device=DEV))
    lg = logits.clone()
    loss = Fn.xent_fwd_bwd(lg, labels, 1.0)
    _close(loss, ref_loss, tol=1e-3)
    _close(lg, g, tol=1e-2)


def test_embedding_fwd_bwd_deterministic():
    torch.manual_seed(10)
    V, H, T = 4096, 1024, 5000
    W = _bf(V, H)
    ids = torch.randint(0, V, (T,), device=DEV, dtype=torch.int32)
    out = Fn.embedding_fwd(W, ids)
    assert torch.equal(out, W[ids.long()])
    dout = _bf(T, H)
    d1 = torch.zeros(V, H, device=DEV)
    d2 = torch.zeros(V, H, device=DEV)
    Fn.embedding_bwd(dout, ids, d1)
    Fn.embedding_bwd(dout, ids, d2)
    assert torch.equal(d1, d2)
    expect = torch.zeros(V, H, device=DEV).index_add_(0, ids.long(), dout.float())
    _close(d1, expect, tol=1e-5)


def test_swiglu_kernels():
    torch.manual_seed(11)
    R, F = 300, 672
    h = _bf(R, 2 * F)
    a = Fn.swiglu_fwd(h)
    _close(a, ref.swiglu_interleaved(h.float()))
    da = _bf(R, F)
    dh = Fn.swiglu_bwd(h, da)
    (g,) = ref.grad_of(ref.swiglu_interleaved, [h.float()], da.float())
    _close(dh, g)


def test_adamw_matches_torch():
    torch.manual_seed(12)
    n = 10_007
    master = torch.randn(n, device=DEV)
    m = torch.randn(n, device=DEV).abs() * 0.01
    v = torch.randn(n, device=DEV).abs() * 0.001
    g1, g2 = _bf(n), _bf(n)
    outs = [torch.empty_like(master) for _ in range(3)]
    pb = torch.empty(n, device=DEV, dtype=torch.bfloat16)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    Fn.adamw_step(master, m, v, [g1, g2], *outs, pb, 1e-3, 0.9, 0.999, 1e-8, 0.01, 7, 0.5, flag)
    g = (g1.float() + g2.float()) * 0.5
    em, emm, ev = ref.adamw(master, m, v, g, 1e-3, 0.9, 0.999, 1e-8, 0.01, 7)
    # fp32 arithmetic; differences come only from FMA contraction
    _close(outs[0], em, tol=1e-5)
    _close(outs[1], emm, tol=1e-5)
    _close(outs[2], ev, tol=1e-4)
    assert int(flag) == 0
    g1[5] = float("inf")
    Fn.adamw_step(master, m, v, [g1], *outs, pb, 1e-3, 0.9, 0.999, 1e-8, 0.01, 7, 1.0, flag)
    assert int(flag) == 1


def test_adamw_device_step_block_matches_host_scalars():
    """The graph-replayable form (lr and bias corrections read from a device
    block) gives the same bits as the host-scalar form."""
    from shift_b200.engine import StepBlock
    torch.manual_seed(13)
    n = 65_539
    master = torch.randn(n, device=DEV)
    m = torch.randn(n, device=DEV).abs() * 0.01
    v = torch.randn(n, device=DEV).abs() * 0.001
    g1 = _bf(n)
    a = [torch.empty_like(master) for _ in range(3)] + [torch.empty(n, device=DEV, dtype=torch.bfloat16)]
    b = [torch.empty_like(t) for t in a]
    Fn.adamw_step(master, m, v, [g1], *a, 3e-4, 0.9, 0.999, 1e-8, 0.01, 11, 1.0)
    blk = StepBlock(torch.device(DEV))
    blk.write(0, 3e-4, 0.9, 0.999, 11)
    Fn.adamw_step(master, m, v, [g1], *b, 123.0, 0.9, 0.999, 1e-8, 0.01, 1, 1.0, step_dev=blk.dev)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_gemm_tensor_parallel_forms_single_gpu():
    """The exchange forms of the GEMM on one GPU (the 'peer' buffers are
    local tensors): rows of the peer half go to the peer buffer, the rest to
    out; the rotated tile order changes nothing; the in-kernel wait passes on
    a set flag; the last CTA signals with the step tag."""
    from shift_b200.engine import StepBlock
    torch.manual_seed(21)
    T, N, K = 1024, 768, 512
    half = T // 2
    x, w = _bf(T, K), _bf(N, K)
    ref_y = x.float() @ w.float().t()
    blk = StepBlock(torch.device(DEV))
    blk.write(5, 1e-4, 0.9, 0.999, 1)
    flags = torch.zeros(8, dtype=torch.int32, device=DEV)
    flags[0] = 5                                    # the "peer" has published its rows
    for rank in (0, 1):
        own = slice(rank * half, (rank + 1) * half)
        plo, phi = (1 - rank) * half, (2 - rank) * half
        out = torch.zeros(half, N, dtype=torch.bfloat16, device=DEV)
        peer = torch.zeros(half, N, dtype=torch.bfloat16, device=DEV)
        xc = [flags[0].data_ptr(), 0, flags[1 + rank].data_ptr(), flags[4 + rank].data_ptr(), 0,
              blk.dev.data_ptr(), peer.data_ptr()]
        G.linear_fwd(x, w, out=out, xchg=xc, tp=(plo, phi, (plo // 128), plo, phi, own.start))
        torch.cuda.synchronize()
        check_status()
        _close(out, ref_y[own])
        _close(peer, ref_y[plo:phi])
        assert int(flags[1 + rank]) == 5 and int(flags[4 + rank]) == 0   # signalled, counter reset
    # k-mode (weight gradient) with a wait over the peer's token rows
    dy = _bf(T, N)
    dw = torch.empty(N, K, dtype=torch.bfloat16, device=DEV)
    G.linear_wgrad(dy, x, dw, xchg=[flags[0].data_ptr(), 0, 0, 0, 0, blk.dev.data_ptr(), 0], tp=(half, T, 0, 0, 0, 0))
    torch.cuda.synchronize()
    check_status()
    _close(dw, dy.float().t() @ x.float())


def test_norm_exchange_forms_single_gpu():
    """RMSNorm fwd/bwd with a second partial (delta2 / dy2), an explicit
    output buffer and a copy into a 'peer' buffer, signalled with the tag."""
    from shift_b200.engine import StepBlock
    torch.manual_seed(22)
    T, H = 512, 1024
    x, d1, d2 = _bf(T, H), _bf(T, H), _bf(T, H)
    w = _bf(H, std=0.1) + 1
    blk = StepBlock(torch.device(DEV))
    blk.write(9, 1e-4, 0.9, 0.999, 1)
    flags = torch.zeros(8, dtype=torch.int32, device=DEV)
    flags[0] = 9
    y_out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    y_peer = torch.empty_like(y_out)
    xc = [flags[0].data_ptr(), 0, flags[1].data_ptr(), flags[2].data_ptr(), 0, blk.dev.data_ptr(), y_peer.data_ptr()]
    y, rstd, h = Fn.rmsnorm_fwd(x, w, 1e-6, d1, delta2=d2, y_out=y_out, xchg=xc)
    torch.cuda.synchronize()
    check_status()
    hr = (x.float() + d1.float() + d2.float()).to(torch.bfloat16)
    assert torch.equal(h, hr)
    _close(y_out, ref.rmsnorm(hr.float(), w.float(), 1e-6))
    assert torch.equal(y_out, y_peer) and int(flags[1]) == 9
    dy, dy2, dres = _bf(T, H), _bf(T, H), _bf(T, H)
    dw = torch.zeros(H, device=DEV)
    dx_out = torch.empty_like(y_out)
    dx_peer = torch.empty_like(y_out)
    xc = [flags[0].data_ptr(), 0, flags[3].data_ptr(), flags[4].data_ptr(), 0, blk.dev.data_ptr(), dx_peer.data_ptr()]
    Fn.rmsnorm_bwd(dy, h, rstd, w, 1e-6, dw, dres=dres, dy2=dy2, dx_out=dx_out, xchg=xc)
    torch.cuda.synchronize()
    check_status()
    dsum = dy.float() + dy2.float()
    (gx, gw) = ref.grad_of(lambda a, b: ref.rmsnorm(a, b, 1e-6), [h.float(), w.float()], dsum)
    _close(dx_out, gx + dres.float())
    _close(dw, gw)
    assert torch.equal(dx_out, dx_peer) and int(flags[3]) == 9



def test_grouped_dgrad_with_swiglu_backward_epilogue():
    """dh = swiglu'(h) . (dy @ w2) computed in the dgrad epilogue equals the
    two-step form (dgrad, then the SwiGLU backward kernel)."""
    torch.manual_seed(23)
    counts = [200, 0, 130, 256]
    offs = _offsets(counts)
    R = int(offs[-1])
    Gn, H, F = len(counts), 1024, 672
    dy = _bf(R, H)
    w2 = _bf(Gn, H, F, std=0.05)
    h = _bf(R, 2 * F)
    dh = G.grouped_dgrad_swiglu(dy, w2, offs, h)
    ref_dh = Fn.swiglu_bwd(h, G.grouped_dgrad(dy, w2, offs))
    torch.cuda.synchronize()
    check_status()
    o = offs.tolist()
    for g in range(Gn):
        s, e = o[g], o[g + 1]
        if e > s:
            _close(dh[s:e], ref_dh[s:e])

