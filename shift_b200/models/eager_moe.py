"""The benchmark MoE written with stock PyTorch: the in-box baseline path.

Same architecture and math contract as ``QwenMoE`` (Qwen-style MoE: RMSNorm,
fused QKV projection, RoPE, causal GQA attention, router softmax + top-k with
renormalised weights and the load-balancing auxiliary loss, SwiGLU experts,
untied LM head, mean token cross-entropy; fp32 master weights, bf16 compute,
AdamW), but built only from what a plain PyTorch training script uses:

* ``nn.Linear`` / ``torch.matmul`` under ``torch.autocast(bfloat16)`` -- cuBLAS;
* ``F.scaled_dot_product_attention`` (causal, GQA) -- the library attention
  backends (cuDNN / flash);
* ``F.rms_norm``, ``torch.topk``, ``torch.softmax`` and a loop over the
  experts on token rows sorted by expert, as Hugging Face MoE blocks do;
* ``torch.optim.AdamW(fused=True)`` on fp32 parameters, and for more than one
  GPU ``DistributedDataParallel`` (bucketed NCCL all-reduce overlapped with
  backward).

The reference trains the same kind of model through FLASH / Megatron modules
on NCCL and cuBLAS (shift_full/train.py:180-230 builds the model, the DDP
wrapper and ``torch.optim.AdamW``); those packages are not in this image, so
this path stands for "the stock NCCL + cuBLAS build" on the same B200s and
the same configuration (``bench.py --impl eager``).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .qwen_moe import MoEConfig


def _rope_tables(max_pos: int, dim: int, theta: float, device=None):
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, device=device, dtype=torch.float32) / dim))
    ang = torch.outer(torch.arange(max_pos, device=device, dtype=torch.float32), inv)
    return torch.cos(ang), torch.sin(ang)


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, heads, S, D] with rotate-half pairing (d, d + D/2)."""
    S = x.shape[-2]
    c, s = cos[:S].to(x.dtype), sin[:S].to(x.dtype)
    x1, x2 = x.chunk(2, dim=-1)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


class EagerBlock(nn.Module):
    def __init__(self, cfg: MoEConfig):
        super().__init__()
        H, D, F_ = cfg.hidden, cfg.head_dim, cfg.expert_ffn
        self.cfg = cfg
        self.ln1 = nn.Parameter(torch.ones(H))
        self.qkv = nn.Linear(H, (cfg.heads + 2 * cfg.kv_heads) * D, bias=False)
        self.o = nn.Linear(cfg.heads * D, H, bias=False)
        self.ln2 = nn.Parameter(torch.ones(H))
        self.router = nn.Linear(H, cfg.experts, bias=False)
        self.w1 = nn.Parameter(torch.empty(cfg.experts, 2 * F_, H))     # gate rows, then up rows
        self.w2 = nn.Parameter(torch.empty(cfg.experts, H, F_))

    def forward(self, x: torch.Tensor, cos, sin):
        cfg = self.cfg
        B, S, H = x.shape
        D, Hq, Hkv = cfg.head_dim, cfg.heads, cfg.kv_heads
        a = F.rms_norm(x, (H,), self.ln1, cfg.eps)
        qkv = self.qkv(a)
        q, k, v = qkv.split([Hq * D, Hkv * D, Hkv * D], dim=-1)
        # contiguous [B, heads, S, D] operands, as the fused SDPA backends want
        # them (a strided V sends SDPA to its unfused math fallback)
        q = _rope(q.view(B, S, Hq, D).transpose(1, 2), cos, sin).contiguous()
        k = _rope(k.view(B, S, Hkv, D).transpose(1, 2), cos, sin).contiguous()
        v = v.view(B, S, Hkv, D).transpose(1, 2).contiguous()
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=1.0 / math.sqrt(D), enable_gqa=True)
        x = x + self.o(o.transpose(1, 2).reshape(B, S, Hq * D))
        m = F.rms_norm(x, (H,), self.ln2, cfg.eps).reshape(B * S, H)
        probs = torch.softmax(self.router(m).float(), dim=-1)
        top, idx = torch.topk(probs, cfg.top_k, dim=-1)
        w = top / top.sum(-1, keepdim=True) if cfg.norm_topk else top
        # token rows sorted by expert, one GEMM pair per expert
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)
        counts = torch.bincount(flat, minlength=cfg.experts).tolist()
        rows = m[order // cfg.top_k]
        outs = []
        lo = 0
        for e, n in enumerate(counts):
            if n:
                h = rows[lo:lo + n] @ self.w1[e].t()
                g, u = h.chunk(2, dim=-1)
                outs.append((F.silu(g) * u) @ self.w2[e].t())
            lo += n
        y = torch.cat(outs) * w.reshape(-1)[order, None].to(outs[0].dtype)
        moe = torch.zeros_like(m, dtype=y.dtype).index_add_(0, order // cfg.top_k, y)
        x = x + moe.view(B, S, H)
        aux = None
        if cfg.aux_coef > 0:
            frac = torch.bincount(flat, minlength=cfg.experts).float() / float(flat.numel())
            aux = cfg.aux_coef * cfg.experts * (frac * probs.mean(0)).sum()
        return x, aux


class EagerMoE(nn.Module):
    def __init__(self, cfg: MoEConfig, seed: int = 0):
        super().__init__()
        self.cfg = cfg
        H = cfg.hidden
        self.embed = nn.Embedding(cfg.vocab, H)
        self.layers = nn.ModuleList(EagerBlock(cfg) for _ in range(cfg.layers))
        self.norm = nn.Parameter(torch.ones(H))
        self.lm_head = nn.Linear(H, cfg.vocab, bias=False)
        g = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            for name, p in self.named_parameters():
                if p.dim() >= 2:
                    p.copy_(torch.randn(p.shape, generator=g) * cfg.init_std)
        cos, sin = _rope_tables(cfg.max_seq, cfg.head_dim, cfg.rope_theta)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)

    def forward(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        """Mean token loss + auxiliary router loss; tokens / labels [B, S]."""
        x = self.embed(tokens)
        aux_total = 0.0
        for layer in self.layers:
            x, aux = layer(x, self.cos, self.sin)
            if aux is not None:
                aux_total = aux_total + aux
        y = F.rms_norm(x, (self.cfg.hidden,), self.norm, self.cfg.eps)
        logits = self.lm_head(y)
        loss = F.cross_entropy(logits.float().view(-1, self.cfg.vocab), labels.reshape(-1))
        return loss + aux_total


class EagerTrainer:
    """One replica of the eager baseline: bf16 autocast forward / backward on
    fp32 parameters, fused AdamW; with ``world > 1`` the model is wrapped in
    DistributedDataParallel (NCCL)."""

    def __init__(self, cfg: MoEConfig, device: torch.device, lr: float = 3e-4, ddp: bool = False, seed: int = 0):
        self.device = device
        self.model = EagerMoE(cfg, seed).to(device)
        self.net = self.model
        if ddp:
            from torch.nn.parallel import DistributedDataParallel
            self.net = DistributedDataParallel(self.model, device_ids=[device.index], bucket_cap_mb=64,
                                               gradient_as_bucket_view=True)
        self.opt = torch.optim.AdamW(self.model.parameters(), lr=lr, betas=(0.9, 0.95), eps=1e-8,
                                     weight_decay=0.1, fused=device.type == "cuda")

    def step(self, tokens: torch.Tensor, labels: torch.Tensor) -> torch.Tensor:
        self.opt.zero_grad(set_to_none=True)
        with torch.autocast(self.device.type, dtype=torch.bfloat16):
            loss = self.net(tokens, labels)
        loss.backward()
        self.opt.step()
        return loss.detach()


class EagerRunner:
    """``bench.py --impl eager``: the benchmark workload (global batch split
    evenly over the ranks, data parallel only) on the eager baseline, with the
    runner interface the benchmark drives (``step``, ``step_e2e``, ``close``)."""

    def __init__(self, cfg: MoEConfig, device: torch.device, batch: int, seq: int, world: int = 1, rank: int = 0):
        from ..engine import synthetic_batch
        if batch % world:
            raise ValueError("global batch must split evenly over the ranks")
        self.cfg = cfg
        self.device = device
        per = batch // world
        sl = slice(rank * per, (rank + 1) * per)
        self.trainer = EagerTrainer(cfg, device, ddp=world > 1)
        self.dev_batches = [synthetic_batch(cfg, i, batch, seq)[sl].long().to(device) for i in range(2)]
        self.host = synthetic_batch(cfg, 10_000, batch, seq)[sl].long().contiguous().pin_memory()
        self.layout = (f"dp{world} (PyTorch eager baseline: cuBLAS GEMMs under bf16 autocast, SDPA attention, "
                       f"per-expert GEMM loop, fused torch AdamW" + (", DDP NCCL all-reduce)" if world > 1 else ")"))

    def step(self, i: int) -> torch.Tensor:
        d = self.dev_batches[i % len(self.dev_batches)]
        return self.trainer.step(d[:, :-1], d[:, 1:])

    def step_e2e(self, i: int):
        d = self.host.to(self.device, non_blocking=True)
        loss = self.trainer.step(d[:, :-1], d[:, 1:])
        return float(loss.item()), self.host.numel() * self.host.element_size(), 4

    def close(self):
        torch.cuda.synchronize(self.device)
