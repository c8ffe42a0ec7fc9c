"""Tensor parallelism over peer memory (TPPeer) on two GPUs: the fused
all-gather / reduce-scatter kernels give the single-GPU model's loss and
gradients (bf16 tolerance), and the same values as the NCCL backend."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cfg():
    from shift_b200.models.qwen_moe import MoEConfig
    return MoEConfig(vocab=512, hidden=256, layers=2, heads=4, kv_heads=2, head_dim=64, experts=8, top_k=2,
                     expert_ffn=256, max_seq=1024)


def _shard(cfg, W, name, t, tp=2):
    D = cfg.head_dim
    hq, hkv = cfg.heads // tp, cfg.kv_heads // tp
    e_per = cfg.experts // tp
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


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from datetime import timedelta

    from shift_b200.engine import Engine, synthetic_batch
    from shift_b200.models.qwen_moe import Partition
    from shift_b200.ops._ext import status_word
    from shift_b200.parallel.symmetric import SymmetricHeap
    from shift_b200.parallel.tp import TPComm, TPPeer
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        cfg = _cfg()
        B, S = 1, 512
        data = synthetic_batch(cfg, 5, B, S).to(dev)
        tok, lab = data[:, :-1].contiguous(), data[:, 1:].contiguous()
        full = Engine(cfg, dev, bucket_numel=1 << 20)
        W = full.store.model_state_dict()
        part = Partition(expert_lo=rank * 4, expert_hi=(rank + 1) * 4, tp_size=2)
        heap = SymmetricHeap(dist.distributed_c10d._get_default_store(), f"t{rank}", dev)
        peer = TPPeer(dist.group.WORLD, rank, 2, dev, heap, f"t{1 - rank}", tokens=B * S, hidden=cfg.hidden,
                      layers=range(cfg.layers), microbatches=1, timeout_s=20)
        results = {}
        for backend in ("peer", "nccl"):
            comm = peer if backend == "peer" else TPComm(dist.group.WORLD, rank, 2, dev)
            eng = Engine(cfg, dev, part=part, bucket_numel=1 << 20, tp=comm)
            for name in eng.store.offsets:
                eng.store.w(name).copy_(_shard(cfg, W, name, rank))
            if backend == "peer":
                dist.barrier()
                peer.connect(eng.step_block.dev)
                peer.set_slot(0, 0)
            eng.prepare_step(1)
            loss = eng.forward_backward([(tok, lab)], B, S)
            torch.cuda.synchronize()
            results[backend] = (float(loss), {n: eng.store.g(n).float().cpu() for n in eng.store.offsets})
            dist.barrier()
        st = int(status_word(dev)[0])
        if rank == 0:
            lf = float(full.forward_backward([(tok, lab)], B, S))
            q.put(("full", lf, {n: full.store.g(n).float().cpu() for n in W}))
        q.put((rank, results, st))
        dist.barrier()
        heap.close_peers()
    finally:
        dist.destroy_process_group()


def _assemble(cfg, name, grads, g_full):
    D = cfg.head_dim
    hq, hkv = cfg.heads // 2, cfg.kv_heads // 2
    if name.endswith("mlp.w1") or name.endswith("mlp.w2"):
        return torch.cat([grads[0][name], grads[1][name]], 0)
    if name.endswith("attn.o"):
        return torch.cat([grads[t][name].view(g_full.shape[0], hq, D) for t in range(2)], 1).reshape(g_full.shape)
    if name.endswith("attn.qkv"):
        parts = []
        for lo, hi in ((0, hq * D), (hq * D, (hq + hkv) * D), ((hq + hkv) * D, (hq + 2 * hkv) * D)):
            parts += [grads[t][name][lo:hi] for t in range(2)]
        return torch.cat(parts[0:2] + parts[2:4] + parts[4:6], 0)
    return grads[0][name] + grads[1][name]


def test_tp2_peer_memory_matches_single_gpu_and_nccl():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world + 1):
        item = q.get(timeout=300)
        got[item[0]] = item
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert got[0][2] == 0 and got[1][2] == 0, "kernel status word reports a timeout"
    cfg = _cfg()
    lf, gfull = got["full"][1], got["full"][2]
    for backend in ("peer", "nccl"):
        losses = [got[t][1][backend][0] for t in range(2)]
        assert abs(sum(losses) - lf) < 2e-2 * max(1.0, abs(lf)), (backend, losses, lf)
        grads = [got[t][1][backend][1] for t in range(2)]
        for name, g in gfull.items():
            a = _assemble(cfg, name, grads, g).reshape(-1)
            b = g.reshape(-1)
            if b.abs().max() < 1e-7:
                continue
            cos = float(torch.dot(a, b) / (a.norm() * b.norm() + 1e-12))
            assert cos > 0.99, (backend, name, cos)
    # the two backends differ only in where partial sums are rounded
    lp = sum(got[t][1]["peer"][0] for t in range(2))
    ln = sum(got[t][1]["nccl"][0] for t in range(2))
    assert abs(lp - ln) < 1e-2 * max(1.0, abs(ln))
