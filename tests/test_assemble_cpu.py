"""Whole-model weights regenerated from the per-shard seeds equal, once split
again by TP rank, what every rank of a TP2 x PP2 replica initialises."""
import torch

from shift_b200.models.qwen_moe import MoEConfig, Partition, param_specs
from shift_b200.parallel.assemble import initial_model_parallel_weights, is_tp_sharded, merge_tp, shard_seed
from shift_b200.parallel.flat import FlatParams


def _split(cfg, name, full, t, tp=2):
    D, hq, hkv = cfg.head_dim, cfg.heads // tp, cfg.kv_heads // tp
    if name.endswith("attn.qkv"):
        q = full[: cfg.heads * D].view(cfg.heads, D, -1)[t * hq:(t + 1) * hq]
        k = full[cfg.heads * D:(cfg.heads + cfg.kv_heads) * D].view(cfg.kv_heads, D, -1)[t * hkv:(t + 1) * hkv]
        v = full[(cfg.heads + cfg.kv_heads) * D:].view(cfg.kv_heads, D, -1)[t * hkv:(t + 1) * hkv]
        return torch.cat([x.reshape(-1, full.shape[1]) for x in (q, k, v)], 0)
    if name.endswith("attn.o"):
        return full.view(full.shape[0], cfg.heads, D)[:, t * hq:(t + 1) * hq].reshape(full.shape[0], -1)
    if name.endswith("mlp.w1") or name.endswith("mlp.w2"):
        e = cfg.experts // tp
        return full[t * e:(t + 1) * e]
    return full


def test_regenerated_weights_match_every_shard():
    cfg = MoEConfig(vocab=512, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2,
                    expert_ffn=256, max_seq=512)
    full = initial_model_parallel_weights(cfg, tp=2, pp=2)
    lps = cfg.layers // 2
    seen = set()
    for s in range(2):
        for t in range(2):
            part = Partition(layer_lo=s * lps, layer_hi=(s + 1) * lps, has_embed=s == 0, has_head=s == 1,
                             expert_lo=t * 4, expert_hi=(t + 1) * 4, tp_size=2)
            specs = param_specs(cfg, part)
            specs = [x for x in specs if not is_tp_sharded(x.name)] + [x for x in specs if is_tp_sharded(x.name)]
            fp = FlatParams(specs, "cpu", torch.bfloat16, 1 << 20)
            fp.init_(cfg.init_std, seed_of=lambda sp, t=t: shard_seed(sp.name, t))
            for name in fp.offsets:
                assert torch.equal(fp.w(name).float(), _split(cfg, name, full[name], t).float()), name
                seen.add(name)
    assert seen == set(full)
    # merge_tp is the inverse of the split
    name = "layers.0.attn.qkv"
    assert torch.equal(merge_tp(cfg, name, [_split(cfg, name, full[name], t) for t in range(2)]), full[name])
