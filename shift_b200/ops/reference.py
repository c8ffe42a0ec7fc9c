"""Plain fp32 PyTorch statements of every op of the model.

These are the numerical oracle of the kernel tests and the compute path for
CPU tensors (the CPU/gloo fault-tolerance harness).  Backward passes of the
CPU path re-run these forwards under autograd (``grad_of``), so each op has a
single definition.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    rs = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * rs * w.float()).to(x.dtype)


def rope_tables(max_pos: int, head_dim: int, theta: float, device=None):
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float64) / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(pos, inv)
    return ang.cos().float().to(device), ang.sin().float().to(device)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, S: int) -> torch.Tensor:
    """x: [T, H, D] with T = B*S; rotate-half convention."""
    T, H, D = x.shape
    pos = torch.arange(T, device=x.device) % S
    c = cos[pos][:, None, :]
    s = sin[pos][:, None, :]
    x1, x2 = x[..., : D // 2].float(), x[..., D // 2:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, B: int, S: int, scale: float) -> torch.Tensor:
    """Causal GQA attention.  q [T, Hq, D], k/v [T, Hkv, D] -> [T, Hq, D]."""
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    g = Hq // Hkv
    qf = q.float().view(B, S, Hq, D).transpose(1, 2)
    kf = k.float().view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(g, dim=1)
    vf = v.float().view(B, S, Hkv, D).transpose(1, 2).repeat_interleave(g, dim=1)
    s = torch.matmul(qf, kf.transpose(-1, -2)) * scale
    mask = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
    s = s.masked_fill(mask, float("-inf"))
    p = torch.softmax(s, dim=-1)
    o = torch.matmul(p, vf)
    return o.transpose(1, 2).reshape(T, Hq, D).to(q.dtype)


def router(x: torch.Tensor, wr: torch.Tensor, k: int, normalize: bool):
    logits = x.float() @ wr.float().t()
    probs = torch.softmax(logits, dim=-1)
    # deterministic top-k: highest prob first, ties to the lower expert index
    order = torch.argsort(-probs, dim=-1, stable=True)[:, :k]
    sel = torch.gather(probs, 1, order)
    w = sel / sel.sum(-1, keepdim=True) if normalize else sel
    return probs, order.to(torch.int32), w


def swiglu_interleaved(h: torch.Tensor) -> torch.Tensor:
    """h: [R, 2F] with blocks of 16 gate then 16 up columns."""
    R, F2 = h.shape
    hv = h.float().view(R, F2 // 32, 2, 16)
    g, u = hv[:, :, 0, :], hv[:, :, 1, :]
    return (F.silu(g) * u).reshape(R, F2 // 2).to(h.dtype)


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[F, H] gate and up -> [2F, H] rows in blocks of 16 gate / 16 up."""
    Fd, H = gate.shape
    return torch.stack([gate.view(Fd // 16, 16, H), up.view(Fd // 16, 16, H)], dim=1).reshape(2 * Fd, H)


def moe_experts(x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor,
                e_lo: int = 0) -> torch.Tensor:
    """Reference MoE: x [T, H], idx/w [T, k], w1 [E, 2F, H] (interleaved), w2 [E, H, F].
    Only experts [e_lo, e_lo + E) contribute."""
    T, H = x.shape
    E = w1.shape[0]
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    for e in range(E):
        tok, slot = torch.nonzero(idx == (e + e_lo), as_tuple=True)
        if tok.numel() == 0:
            continue
        h = x[tok].float() @ w1[e].float().t()
        a = swiglu_interleaved(h)
        y = a.float() @ w2[e].float().t()
        out.index_add_(0, tok, y * w[tok, slot].float()[:, None])
    return out.to(x.dtype)


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
    return F.cross_entropy(logits.float(), labels.long(), reduction="none", ignore_index=-100)


def adamw(master, m, v, grad, lr, beta1, beta2, eps, wd, step):
    """torch.optim.AdamW single-tensor arithmetic, fp32."""
    master = master * (1 - lr * wd)
    m = m.lerp(grad, 1 - beta1)
    v = v * beta2 + (1 - beta2) * grad * grad
    bc1 = 1 - beta1 ** step
    bc2 = 1 - beta2 ** step
    denom = (v.sqrt() / math.sqrt(bc2)) + eps
    master = master - (lr / bc1) * (m / denom)
    return master, m, v


def grad_of(fn, inputs, grad_out):
    """Gradients of fn(*inputs) w.r.t. the floating inputs, via autograd."""
    # cloned: an input may be a view of a buffer another rank's thread writes
    # into meanwhile (tensor-parallel emulation), which autograd would reject
    leaves = [t.detach().clone().requires_grad_(t.is_floating_point()) if isinstance(t, torch.Tensor) else t
              for t in inputs]
    with torch.enable_grad():
        out = fn(*leaves)
    diff = [t for t in leaves if isinstance(t, torch.Tensor) and t.requires_grad]
    grads = torch.autograd.grad(out, diff, grad_out, allow_unused=True)
    it = iter(grads)
    res = []
    for t in leaves:
        if isinstance(t, torch.Tensor) and t.requires_grad:
            g = next(it)
            res.append(torch.zeros_like(t) if g is None else g)
        else:
            res.append(None)
    return res
