"""Whole-model weights from tensor-parallel shards.

A TP rank holds, of each layer, the query/key/value heads and output-
projection columns of its head range and the experts of its expert range;
everything else is replicated.  ``merge_tp`` inverts that split for one
parameter (the inverse of the head / expert partition done by
``models.qwen_moe.param_specs`` with ``tp_size > 1``), and
``initial_model_parallel_weights`` rebuilds the initial whole-model weights
of a TP x PP replica on the host from the per-parameter seeds the model-
parallel runner initialises with -- so a one-GPU recomputation of the same
step can start from exactly those weights without moving any shard.
"""
from __future__ import annotations

import zlib

import torch

from ..models.qwen_moe import TP_SHARDED, MoEConfig, Partition, param_specs


def is_tp_sharded(name: str) -> bool:
    return any(name.endswith(s) for s in TP_SHARDED)


def shard_seed(name: str, tp_rank: int) -> int:
    """Seed of one parameter's N(0, std) initialisation on TP rank ``tp_rank``
    (replicated parameters get the same seed on every rank)."""
    salt = f"/tp{tp_rank}" if is_tp_sharded(name) else ""
    return 2026 + zlib.crc32((name + salt).encode())


def merge_tp(cfg: MoEConfig, name: str, shards: list) -> torch.Tensor:
    """Whole tensor of parameter ``name`` from its per-TP-rank shards."""
    tp = len(shards)
    if not is_tp_sharded(name):
        return shards[0]
    D = cfg.head_dim
    hq, hkv = cfg.heads // tp, cfg.kv_heads // tp
    if name.endswith("attn.qkv"):
        q = [s[: hq * D] for s in shards]
        k = [s[hq * D:(hq + hkv) * D] for s in shards]
        v = [s[(hq + hkv) * D:] for s in shards]
        return torch.cat(q + k + v, 0)
    if name.endswith("attn.o"):
        return torch.cat(shards, 1)
    return torch.cat(shards, 0)           # experts (mlp.w1 / mlp.w2)


def _initial_value(spec, seed: int, std: float) -> torch.Tensor:
    """The fp32 value ``FlatParams.init_`` gives one parameter."""
    if spec.init == "ones":
        return torch.ones(spec.shape)
    if spec.init == "zeros":
        return torch.zeros(spec.shape)
    t = torch.empty(spec.shape, dtype=torch.float32)
    t.normal_(0.0, std, generator=torch.Generator().manual_seed(seed))
    return t


def initial_model_parallel_weights(cfg: MoEConfig, tp: int, pp: int, dtype=torch.bfloat16) -> dict:
    """{name: whole tensor} of the initial weights of one TP x PP replica of the
    model-parallel runner, rounded to ``dtype`` as the runner's parameters are."""
    lps = cfg.layers // pp
    e_per = cfg.experts // tp
    pieces: dict = {}
    for s in range(pp):
        for t in range(tp):
            part = Partition(layer_lo=s * lps, layer_hi=(s + 1) * lps, has_embed=s == 0, has_head=s == pp - 1,
                             expert_lo=t * e_per, expert_hi=(t + 1) * e_per, tp_size=tp)
            for spec in param_specs(cfg, part):
                if t > 0 and not is_tp_sharded(spec.name):
                    continue
                v = _initial_value(spec, shard_seed(spec.name, t), cfg.init_std).to(dtype)
                pieces.setdefault(spec.name, [None] * tp)[t] = v
    return {n: merge_tp(cfg, n, [p for p in ps if p is not None]) for n, ps in pieces.items()}
