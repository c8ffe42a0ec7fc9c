"""Forward / backward pairs of the non-GEMM ops.

CUDA tensors run the sm_100a kernels of ``shift_b200._C`` (raising if the
extension is absent); CPU tensors run the fp32 statements of
``shift_b200.ops.reference`` (backward by autograd over the same statement).
"""
from __future__ import annotations

import torch

from . import reference as ref
from ._ext import ext, status_word


# ----------------------------------------------------------------------------- RMSNorm
def rmsnorm_fwd(x, w, eps, delta=None, delta2=None, y_out=None, xchg=()):
    """Returns (y, rstd, h) where h = x + delta (+ delta2) (or x when delta
    is None).  ``delta2``/``y_out``/``xchg``: tensor-parallel forms (CUDA)."""
    if x.is_cuda:
        r = ext().rmsnorm_fwd(x, delta, w, eps, delta2, y_out, list(xchg),
                              status_word(x.device) if xchg else None)
        if delta is None:
            return r[0], r[1], x
        return r[0], r[1], r[2]
    _before(xchg)
    h = x if delta is None else (x.float() + delta.float()).to(x.dtype)
    if delta2 is not None:
        h = (x.float() + delta.float() + delta2.float()).to(x.dtype)
    hf = h.float()
    rstd = torch.rsqrt(hf.pow(2).mean(-1) + eps)
    y = ref.rmsnorm(h, w, eps)
    if y_out is not None:
        y = y_out.copy_(y)
    _after(xchg, y)
    return y, rstd, h


def _before(xchg):
    """CPU stand-ins of the kernels' tensor-parallel exchange hooks."""
    if xchg and hasattr(xchg, "before"):
        xchg.before()


def _after(xchg, peer_rows=None):
    if xchg and hasattr(xchg, "after"):
        if peer_rows is not None and xchg.peer_out is not None:
            xchg.peer_out.copy_(peer_rows)
        xchg.after()


def rmsnorm_bwd(dy, h, rstd, w, eps, dw_out, dres=None, accumulate=False, dy2=None, dx_out=None, xchg=()):
    """dx = d(norm)/dh + dres;  dw_out (+)= dw.  ``dy2``: a second partial of
    dy (tensor-parallel reduce-scatter fused in); ``dx_out``/``xchg``: write
    dx there and copy it into a peer's gather buffer, then signal."""
    if dy.is_cuda:
        return ext().rmsnorm_bwd(dy, h, rstd, w, dres, dw_out, accumulate, dy2, dx_out, list(xchg),
                                 status_word(h.device) if xchg else None)
    _before(xchg)
    if dy2 is not None:
        dy = (dy.float() + dy2.float()).to(dy.dtype)
    dh, dw = ref.grad_of(lambda a, b: ref.rmsnorm(a, b, eps), [h, w], dy)
    if dres is not None:
        dh = dh + dres
    if accumulate:
        dw_out.add_(dw.to(dw_out.dtype))
    else:
        dw_out.copy_(dw)
    dh = dh.to(dy.dtype)
    if dx_out is not None:
        dh = dx_out.copy_(dh)
    _after(xchg, dh)
    return dh


# ----------------------------------------------------------------------------- RoPE
def rope_(qkv, cos, sin, S, n_rot_heads, head_dim, inverse=False):
    """In-place rotary embedding of the first n_rot_heads heads of qkv [T, W]."""
    if qkv.is_cuda:
        ext().rope_(qkv, cos, sin, S, n_rot_heads, head_dim, 0, inverse)
        return qkv
    T = qkv.shape[0]
    part = qkv[:, : n_rot_heads * head_dim].view(T, n_rot_heads, head_dim)
    s = -sin if inverse else sin
    part.copy_(ref.rope(part, cos, s, S))
    return qkv


# ----------------------------------------------------------------------------- attention
def attention_fwd(qkv, B, S, Hq, Hkv, D, scale):
    """Returns (o [T, Hq*D], lse)."""
    if qkv.is_cuda:
        o, lse = ext().attn_fwd(qkv, B, S, Hq, Hkv, scale, status_word(qkv.device))
        return o, lse
    T = qkv.shape[0]
    q = qkv[:, : Hq * D].view(T, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
    v = qkv[:, (Hq + Hkv) * D:].view(T, Hkv, D)
    return ref.attention(q, k, v, B, S, scale).reshape(T, Hq * D), None


def attention_bwd(qkv, o, lse, do, B, S, Hq, Hkv, D, scale):
    if qkv.is_cuda:
        return ext().attn_bwd(qkv, o, lse, do, B, S, Hq, Hkv, scale, status_word(qkv.device))
    T = qkv.shape[0]

    def f(x):
        q = x[:, : Hq * D].view(T, Hq, D)
        k = x[:, Hq * D:(Hq + Hkv) * D].view(T, Hkv, D)
        v = x[:, (Hq + Hkv) * D:].view(T, Hkv, D)
        return ref.attention(q, k, v, B, S, scale).reshape(T, Hq * D)

    (g,) = ref.grad_of(f, [qkv], do)
    return g.to(qkv.dtype)


# ----------------------------------------------------------------------------- router
def router_fwd(x, wr, k, normalize):
    """Returns (probs [T,E] fp32, idx [T,k] int32, w [T,k] fp32)."""
    if x.is_cuda:
        return tuple(ext().router_fwd(x, wr, k, normalize))
    return ref.router(x, wr, k, normalize)


def router_bwd(x, wr, probs, idx, w, dw_topk, aux_grad, normalize, dx, dwr_out, accumulate=False,
               peer_rows=(), xchg=()):
    """dx += d(router)/dx (in place); dwr_out (+)= dWr.  ``peer_rows`` /
    ``xchg`` (CUDA): rows [lo, hi) of the finished dx are stored into the
    tensor-parallel peer's receive buffer instead, then the kernel signals."""
    if x.is_cuda:
        dl = ext().router_bwd(probs, idx, w, dw_topk, aux_grad, normalize)
        partial = ext().router_input_weight_grad(x, wr, dl, dx, list(peer_rows), list(xchg))
        ext().column_reduce(partial, dwr_out.view(-1), accumulate)
        return dx
    _router_bwd_cpu(x, wr, idx, dw_topk, aux_grad, normalize, dx, dwr_out, accumulate)
    if xchg:
        lo, hi = peer_rows
        _after(xchg, dx[lo:hi])
    return dx


def _router_bwd_cpu(x, wr, idx, dw_topk, aux_grad, normalize, dx, dwr_out, accumulate):
    E = wr.shape[0]

    def f(xx, ww):
        logits = xx.float() @ ww.float().t()
        p = torch.softmax(logits, -1)
        sel = torch.gather(p, 1, idx.long())
        wt = sel / sel.sum(-1, keepdim=True) if normalize else sel
        out = (wt * dw_topk).sum()
        if aux_grad is not None:
            out = out + (p * aux_grad[None, :]).sum()
        return out

    gx, gw = ref.grad_of(f, [x, wr], torch.tensor(1.0))
    dx.add_(gx.to(dx.dtype))
    if accumulate:
        dwr_out.add_(gw.to(dwr_out.dtype))
    else:
        dwr_out.copy_(gw)
    del E
    return dx


# ----------------------------------------------------------------------------- permutation
def bucket_sort(keys, lo, hi, pad, src_div):
    """Stable sort of keys into bins [lo, hi).  Returns (pos, offs, counts, row_src)."""
    if keys.is_cuda:
        return tuple(ext().bucket_sort(keys, lo, hi, pad, src_div))
    flat = keys.reshape(-1).long()
    nb = hi - lo
    counts = torch.zeros(nb, dtype=torch.int64)
    valid = (flat >= lo) & (flat < hi)
    for b in range(nb):
        counts[b] = int(((flat == b + lo) & valid).sum())
    padded = ((counts + pad - 1) // pad) * pad if pad > 1 else counts
    offs = torch.zeros(nb + 1, dtype=torch.int64)
    offs[1:] = torch.cumsum(padded, 0)
    cap = flat.numel() + nb * max(0, pad - 1)
    pos = torch.full((flat.numel(),), -1, dtype=torch.int64)
    row_src = torch.full((cap,), -1, dtype=torch.int64)
    fill = offs[:-1].clone()
    for i in range(flat.numel()):
        if valid[i]:
            b = int(flat[i]) - lo
            pos[i] = fill[b]
            row_src[fill[b]] = i // src_div
            fill[b] += 1
    return pos.int(), offs.int(), counts.int(), row_src.int()


def gather_rows(src, row_src, total, cap):
    if src.is_cuda:
        out = torch.empty(cap, src.shape[1], dtype=src.dtype, device=src.device)
        ext().gather_rows(src, row_src, total, out)
        return out
    out = torch.zeros(cap, src.shape[1], dtype=src.dtype)
    valid = row_src[:cap] >= 0
    out[valid] = src[row_src[:cap][valid].long()]
    return out


def combine(y, pos, w, T, out=None, split=(), xchg=()):
    """Weighted sum of each token's expert rows.  ``split`` = (peer_lo,
    peer_hi, own_off) with ``xchg`` (CUDA): token rows [peer_lo, peer_hi) go
    to the tensor-parallel peer's receive buffer, the rest to ``out``."""
    if y.is_cuda:
        return ext().combine(y, pos, w, T, out, list(split), list(xchg))
    full = torch.zeros(T, y.shape[1], dtype=torch.float32)
    k = pos.shape[1]
    for j in range(k):
        p = pos[:, j].long()
        ok = p >= 0
        full[ok] += w[ok, j:j + 1].float() * y[p[ok]].float()
    full = full.to(y.dtype)
    if not split:
        return full
    lo, hi, own_off = split
    keep = torch.ones(T, dtype=torch.bool)
    keep[lo:hi] = False
    out.copy_(full[keep])
    _after(xchg, full[lo:hi])
    return out


def combine_bwd(dout, y, pos, w, row_src, slot_of_row, total):
    """Returns (dy rows, dw [T,k])."""
    if dout.is_cuda:
        return tuple(ext().combine_bwd(dout, y, pos, w, row_src, slot_of_row, total))
    cap = y.shape[0]
    dy = torch.zeros_like(y, dtype=torch.float32)
    k = pos.shape[1]
    dw = torch.zeros(pos.shape, dtype=torch.float32)
    for j in range(k):
        p = pos[:, j].long()
        ok = p >= 0
        dy[p[ok]] = w[ok, j:j + 1].float() * dout[ok].float()
        dw[ok, j] = (dout[ok].float() * y[p[ok]].float()).sum(-1)
    del cap
    return dy.to(y.dtype), dw


def scatter_back(dperm, pos, dx, accumulate):
    if dperm.is_cuda:
        ext().scatter_back(dperm, pos, dx, accumulate)
        return dx
    acc = dx.float() if accumulate else torch.zeros_like(dx, dtype=torch.float32)
    for j in range(pos.shape[1]):
        p = pos[:, j].long()
        ok = p >= 0
        acc[ok] += dperm[p[ok]].float()
    dx.copy_(acc)
    return dx


def invert_pos(pos, cap):
    if pos.is_cuda:
        return ext().invert_pos(pos.reshape(-1).contiguous(), cap)
    out = torch.full((cap,), -1, dtype=torch.int32)
    flat = pos.reshape(-1)
    ok = flat >= 0
    out[flat[ok].long()] = torch.nonzero(ok).reshape(-1).int()
    return out


# ----------------------------------------------------------------------------- SwiGLU
def swiglu_fwd(h):
    if h.is_cuda:
        return ext().swiglu_fwd(h)
    return ref.swiglu_interleaved(h)


def swiglu_bwd(h, da):
    if h.is_cuda:
        return ext().swiglu_bwd(h, da)
    (g,) = ref.grad_of(ref.swiglu_interleaved, [h], da)
    return g.to(h.dtype)


# ----------------------------------------------------------------------------- embedding / loss
def embedding_fwd(W, ids, vocab_lo=0):
    if W.is_cuda:
        return ext().embedding_fwd(W, ids, vocab_lo)
    loc = ids.long() - vocab_lo
    ok = (loc >= 0) & (loc < W.shape[0])
    out = torch.zeros(ids.numel(), W.shape[1], dtype=W.dtype)
    out[ok] = W[loc[ok]]
    return out


def embedding_bwd(dout, ids, dW32, vocab_lo=0):
    """dW32 (fp32 [V, H]) += scattered rows, deterministic."""
    if dout.is_cuda:
        ext().embedding_bwd(dout, ids, dW32, vocab_lo)
        return dW32
    loc = ids.long() - vocab_lo
    ok = (loc >= 0) & (loc < dW32.shape[0])
    dW32.index_add_(0, loc[ok], dout[ok].float())
    return dW32


def xent_fwd_bwd(logits, labels, scale, label_lo=0):
    """Per-row loss; logits are overwritten by scale * dloss/dlogits."""
    if logits.is_cuda:
        return ext().xent_fwd_bwd(logits, labels, scale, label_lo)
    lab = labels.long() - label_lo
    valid = labels >= 0
    lf = logits.float()
    lse = torch.logsumexp(lf, -1)
    picked = torch.gather(lf, 1, lab.clamp(min=0)[:, None])[:, 0]
    loss = torch.where(valid, lse - picked, torch.zeros_like(lse))
    g = torch.softmax(lf, -1)
    g[torch.arange(g.shape[0])[valid], lab[valid]] -= 1.0
    g = g * scale * valid[:, None].float()
    logits.copy_(g.to(logits.dtype))
    return loss


# ----------------------------------------------------------------------------- optimizer
def adamw_step(master, m, v, grads, master_out, m_out, v_out, param_out, lr, beta1, beta2, eps, wd, step,
               grad_scale, nonfinite=None, step_dev=None):
    """``step_dev`` (CUDA only): int32 device block whose [1..3] hold lr,
    1 - beta1^t and sqrt(1 - beta2^t) as float bits; it overrides lr/step."""
    if master.is_cuda:
        ext().adamw_step(master, m, v, list(grads), master_out, m_out, v_out, param_out, lr, beta1, beta2, eps, wd,
                         step, grad_scale, nonfinite, step_dev)
        return
    g = grads[0].float().clone()
    for extra in grads[1:]:
        g += extra.float()
    g *= grad_scale
    if nonfinite is not None and not torch.isfinite(g).all():
        nonfinite.fill_(1)
    p2, m2, v2 = ref.adamw(master, m, v, g, lr, beta1, beta2, eps, wd, step)
    master_out.copy_(p2)
    m_out.copy_(m2)
    v_out.copy_(v2)
    param_out.copy_(p2.to(param_out.dtype))


def nonfinite_check(x, flag):
    if x.is_cuda:
        ext().nonfinite_check(x, flag)
    elif not torch.isfinite(x.float()).all():
        flag.fill_(1)
