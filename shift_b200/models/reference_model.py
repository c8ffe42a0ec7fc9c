"""Autograd statement of the whole MoE loss, built only from the fp32
reference ops.  It is the oracle for the explicit forward/backward of
``QwenMoE`` (CPU tests) and for the CUDA kernels end to end (GPU tests)."""
from __future__ import annotations

import math

import torch

from ..ops import reference as ref
from .qwen_moe import MoEConfig


def reference_loss(cfg: MoEConfig, params: dict, tokens: torch.Tensor, labels: torch.Tensor, B: int, S: int,
                   with_aux: bool = True) -> torch.Tensor:
    """Mean token loss (+ auxiliary router loss) for fp32 leaf tensors ``params``."""
    H, D, Hq, Hkv = cfg.hidden, cfg.head_dim, cfg.heads, cfg.kv_heads
    T = B * S
    cos, sin = ref.rope_tables(cfg.max_seq, D, cfg.rope_theta)
    scale = 1.0 / math.sqrt(D)
    x = params["embed.weight"][tokens.reshape(-1).long()]
    aux_total = 0.0
    for i in range(cfg.layers):
        p = f"layers.{i}."
        a = ref.rmsnorm(x, params[p + "ln1.weight"], cfg.eps)
        qkv = a @ params[p + "attn.qkv"].t()
        q = ref.rope(qkv[:, : Hq * D].reshape(T, Hq, D), cos, sin, S)
        k = ref.rope(qkv[:, Hq * D:(Hq + Hkv) * D].reshape(T, Hkv, D), cos, sin, S)
        v = qkv[:, (Hq + Hkv) * D:].reshape(T, Hkv, D)
        o = ref.attention(q, k, v, B, S, scale).reshape(T, Hq * D)
        x = x + o @ params[p + "attn.o"].t()
        m = ref.rmsnorm(x, params[p + "ln2.weight"], cfg.eps)
        logits = m @ params[p + "mlp.router"].t()
        probs = torch.softmax(logits, -1)
        idx = torch.argsort(-probs.detach(), dim=-1, stable=True)[:, : cfg.top_k]
        sel = torch.gather(probs, 1, idx)
        w = sel / sel.sum(-1, keepdim=True) if cfg.norm_topk else sel
        x = x + ref.moe_experts(m, idx, w, params[p + "mlp.w1"], params[p + "mlp.w2"])
        if with_aux and cfg.aux_coef > 0:
            counts = torch.stack([(idx == e).sum() for e in range(cfg.experts)]).float()
            f = counts / float(T * cfg.top_k)
            aux_total = aux_total + cfg.aux_coef * cfg.experts * (f * probs.mean(0)).sum()
    y = ref.rmsnorm(x, params["norm.weight"], cfg.eps)
    lg = y @ params["lm_head.weight"].t()
    loss = ref.cross_entropy(lg, labels.reshape(-1)).mean()
    return loss + aux_total
