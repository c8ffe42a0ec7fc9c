"""Tensor parallelism (sequence parallel, experts split over the TP pair) on
CPU: two threads run the two TP ranks with an in-process all-gather /
reduce-scatter; loss and gradients must equal the single-rank model's."""
import threading
import zlib

import torch

from shift_b200.engine import Engine, synthetic_batch
from shift_b200.models.qwen_moe import TP_SHARDED, MoEConfig, Partition, param_specs


class ThreadTP:
    """all_gather / reduce_scatter between threads (rank order, fixed-order sums)."""

    def __init__(self, size):
        self.size = size
        self.bar = threading.Barrier(size)
        self.slots = [None] * size

    def view(self, rank):
        outer = self

        class V:
            size = outer.size

            def __init__(self):
                self.rank = rank

            def all_gather(self, x):
                outer.slots[rank] = x.clone()
                outer.bar.wait()
                out = torch.cat(outer.slots, 0)
                outer.bar.wait()
                return out

            def reduce_scatter(self, x):
                outer.slots[rank] = x.clone()
                outer.bar.wait()
                n = x.shape[0] // outer.size
                total = outer.slots[0].float()
                for s in outer.slots[1:]:
                    total = total + s.float()
                out = total[rank * n:(rank + 1) * n].to(x.dtype).clone()
                outer.bar.wait()
                return out

            def all_reduce_(self, x):
                raise NotImplementedError

            def local_rows(self, x):
                n = x.shape[0] // outer.size
                return x[rank * n:(rank + 1) * n]

        return V()


def _cfg():
    return MoEConfig(vocab=512, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2,
                     expert_ffn=256, max_seq=256)


def _sharded(name):
    return any(name.endswith(s) for s in TP_SHARDED)


def test_tp2_matches_single_rank():
    torch.manual_seed(0)
    cfg = _cfg()
    B, S, tp = 1, 128, 2
    data = synthetic_batch(cfg, 11, B, S)
    tok, lab = data[:, :-1].contiguous(), data[:, 1:].contiguous()
    full = Engine(cfg, "cpu", bucket_numel=1 << 20)
    loss_full = float(full.forward_backward([(tok, lab)], B, S))
    W = full.store.model_state_dict()
    comm = ThreadTP(tp)
    engines, losses, errors = [None] * tp, [None] * tp, []
    D = cfg.head_dim
    hq, hkv = cfg.heads // tp, cfg.kv_heads // tp
    e_per = cfg.experts // tp

    def shard_of(name, t):
        w = W[name]
        if name.endswith("attn.qkv"):
            q = w[: cfg.heads * D].view(cfg.heads, D, -1)[t * hq:(t + 1) * hq].reshape(-1, w.shape[1])
            k = w[cfg.heads * D:(cfg.heads + cfg.kv_heads) * D].view(cfg.kv_heads, D, -1)[t * hkv:(t + 1) * hkv]
            v = w[(cfg.heads + cfg.kv_heads) * D:].view(cfg.kv_heads, D, -1)[t * hkv:(t + 1) * hkv]
            return torch.cat([q, k.reshape(-1, w.shape[1]), v.reshape(-1, w.shape[1])], 0)
        if name.endswith("attn.o"):
            return w.view(w.shape[0], cfg.heads, D)[:, t * hq:(t + 1) * hq].reshape(w.shape[0], -1)
        if name.endswith("mlp.w1") or name.endswith("mlp.w2"):
            return w[t * e_per:(t + 1) * e_per]
        return w

    def run(t):
        try:
            part = Partition(expert_lo=t * e_per, expert_hi=(t + 1) * e_per, tp_size=tp)
            eng = Engine(cfg, "cpu", part=part, bucket_numel=1 << 20, tp=comm.view(t))
            for name in eng.store.offsets:
                eng.store.w(name).copy_(shard_of(name, t))
            losses[t] = float(eng.forward_backward([(tok, lab)], B, S))
            engines[t] = eng
        except BaseException as e:  # pragma: no cover - surfaced below
            errors.append(e)
            comm.bar.abort()

    ths = [threading.Thread(target=run, args=(t,)) for t in range(tp)]
    for th in ths:
        th.start()
    for th in ths:
        th.join(120)
    assert not errors, errors
    # each rank reports the loss of its own token half
    assert abs(sum(losses) - loss_full) < 1e-4
    for name, g_full in ((n, full.store.g(n)) for n in W):
        if _sharded(name):
            got = torch.cat([engines[t].store.g(name) for t in range(tp)], 0) if "mlp" in name else None
            if name.endswith("attn.o"):
                got = torch.cat([engines[t].store.g(name).view(g_full.shape[0], hq, D) for t in range(tp)], 1)
                got = got.reshape(g_full.shape)
            if name.endswith("attn.qkv"):
                gq = torch.cat([engines[t].store.g(name)[: hq * D] for t in range(tp)], 0)
                gk = torch.cat([engines[t].store.g(name)[hq * D:(hq + hkv) * D] for t in range(tp)], 0)
                gv = torch.cat([engines[t].store.g(name)[(hq + hkv) * D:] for t in range(tp)], 0)
                got = torch.cat([gq, gk, gv], 0)
        else:
            # replicated parameters: the TP pair's gradients sum to the full gradient
            got = engines[0].store.g(name) + engines[1].store.g(name)
        err = (got - g_full).abs().max().item()
        scale = g_full.abs().max().item() + 1e-8
        assert err <= 2e-4 * max(1.0, scale) + 1e-7, (name, err, scale)


def test_sharded_names_and_seeded_init_are_rank_consistent():
    cfg = _cfg()
    specs0 = param_specs(cfg, Partition(expert_lo=0, expert_hi=4, tp_size=2))
    specs1 = param_specs(cfg, Partition(expert_lo=4, expert_hi=8, tp_size=2))
    assert [s.name for s in specs0] == [s.name for s in specs1]
    seed = lambda t: (lambda s: 2026 + zlib.crc32((s.name + (f"/tp{t}" if _sharded(s.name) else "")).encode()))
    e0 = Engine(cfg, "cpu", part=Partition(expert_lo=0, expert_hi=4, tp_size=2), seed_of=seed(0))
    e1 = Engine(cfg, "cpu", part=Partition(expert_lo=4, expert_hi=8, tp_size=2), seed_of=seed(1))
    for name in e0.store.offsets:
        same = torch.equal(e0.store.w(name), e1.store.w(name))
        assert same == (not _sharded(name)) or "ln" in name, name


def test_tp2_peer_exchange_protocol_matches_single_rank():
    """The symmetric-memory TP path (TPPeer: gather buffers written by the
    producer on both ranks, partial sums stored into the peer's receive
    buffer, flags as events) on CPU threads gives the single-rank result."""
    from shift_b200.parallel.tp import TPPeer

    class Heap:
        def __init__(self, owner):
            self.owner = owner

    torch.manual_seed(0)
    cfg = _cfg()
    B, S, tp = 1, 256, 2
    data = synthetic_batch(cfg, 12, B, S)
    tok, lab = data[:, :-1].contiguous(), data[:, 1:].contiguous()
    full = Engine(cfg, "cpu", bucket_numel=1 << 20)
    loss_full = float(full.forward_backward([(tok, lab)], B, S))
    W = full.store.model_state_dict()
    D = cfg.head_dim
    hq, hkv = cfg.heads // tp, cfg.kv_heads // tp
    e_per = cfg.experts // tp
    bar = threading.Barrier(tp)
    engines, losses, errors = [None] * tp, [None] * tp, []

    def shard_of(name, t):
        w = W[name]
        if name.endswith("attn.qkv"):
            q = w[: cfg.heads * D].view(cfg.heads, D, -1)[t * hq:(t + 1) * hq].reshape(-1, w.shape[1])
            k = w[cfg.heads * D:(cfg.heads + cfg.kv_heads) * D].view(cfg.kv_heads, D, -1)[t * hkv:(t + 1) * hkv]
            v = w[(cfg.heads + cfg.kv_heads) * D:].view(cfg.kv_heads, D, -1)[t * hkv:(t + 1) * hkv]
            return torch.cat([q, k.reshape(-1, w.shape[1]), v.reshape(-1, w.shape[1])], 0)
        if name.endswith("attn.o"):
            return w.view(w.shape[0], cfg.heads, D)[:, t * hq:(t + 1) * hq].reshape(w.shape[0], -1)
        if name.endswith("mlp.w1") or name.endswith("mlp.w2"):
            return w[t * e_per:(t + 1) * e_per]
        return w

    def run(t):
        try:
            peer = TPPeer(None, t, tp, "cpu", Heap(f"cpu_t{t}"), f"cpu_t{1 - t}", tokens=B * S, hidden=cfg.hidden,
                          layers=range(cfg.layers), microbatches=1, timeout_s=60)
            part = Partition(expert_lo=t * e_per, expert_hi=(t + 1) * e_per, tp_size=tp)
            eng = Engine(cfg, "cpu", part=part, bucket_numel=1 << 20, tp=peer)
            for name in eng.store.offsets:
                eng.store.w(name).copy_(shard_of(name, t))
            bar.wait()
            peer.connect(eng.step_block.dev)
            peer.set_slot(0, 0)
            eng.prepare_step(1)
            losses[t] = float(eng.forward_backward([(tok, lab)], B, S))
            engines[t] = eng
        except BaseException as e:  # pragma: no cover - surfaced below
            errors.append(e)
            bar.abort()

    ths = [threading.Thread(target=run, args=(t,)) for t in range(tp)]
    for th in ths:
        th.start()
    for th in ths:
        th.join(300)
    assert not errors, errors
    assert abs(sum(losses) - loss_full) < 1e-4
    for name in W:
        g_full = full.store.g(name)
        if _sharded(name):
            if "mlp" in name:
                got = torch.cat([engines[t].store.g(name) for t in range(tp)], 0)
            elif name.endswith("attn.o"):
                got = torch.cat([engines[t].store.g(name).view(g_full.shape[0], hq, D) for t in range(tp)], 1)
                got = got.reshape(g_full.shape)
            else:
                gq = torch.cat([engines[t].store.g(name)[: hq * D] for t in range(tp)], 0)
                gk = torch.cat([engines[t].store.g(name)[hq * D:(hq + hkv) * D] for t in range(tp)], 0)
                gv = torch.cat([engines[t].store.g(name)[(hq + hkv) * D:] for t in range(tp)], 0)
                got = torch.cat([gq, gk, gv], 0)
        else:
            got = engines[0].store.g(name) + engines[1].store.g(name)
        err = (got - g_full).abs().max().item()
        scale = g_full.abs().max().item() + 1e-8
        assert err <= 2e-4 * max(1.0, scale) + 1e-7, (name, err, scale)
