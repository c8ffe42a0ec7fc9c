"""Peer-memory collectives: K1 (fused cross-replica reduce + AdamW), bounded
flag waits, K10 peer copy.  Multi-GPU cases run as child processes."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from shift_b200.ops import reference as ref
from shift_b200.ops._ext import ext, status_word

pytestmark = pytest.mark.gpu


def _step_block(dev, tag, lr, beta1, beta2, step):
    from shift_b200.engine import StepBlock
    sb = StepBlock(dev)
    sb.write(tag, lr, beta1, beta2, step)
    return sb.dev


def test_fused_reduce_adamw_local_sources_matches_reference():
    torch.manual_seed(0)
    n = 100_003
    dev = torch.device("cuda", 0)
    master = torch.randn(n, device=dev)
    m = torch.randn(n, device=dev) * 0.01
    v = torch.rand(n, device=dev) * 1e-3
    gs = [(torch.randn(n, device=dev)).to(torch.bfloat16) for _ in range(3)]
    outs = [torch.empty_like(master) for _ in range(3)]
    pb = torch.empty(n, device=dev, dtype=torch.bfloat16)
    flag = torch.zeros(1, dtype=torch.int32, device=dev)
    st = status_word(dev)
    st.zero_()
    sdev = _step_block(dev, 1, 1e-3, 0.9, 0.999, 5)
    ext().fused_reduce_adamw([g.data_ptr() for g in gs], [], sdev, master, m, v, *outs, pb, 0.9, 0.999, 1e-8,
                             0.01, 1 / 3, flag, st, 5.0, 0)
    torch.cuda.synchronize()
    g = (gs[0].float() + gs[1].float() + gs[2].float()) / 3
    em, emm, ev = ref.adamw(master, m, v, g, 1e-3, 0.9, 0.999, 1e-8, 0.01, 5)
    assert torch.allclose(outs[0], em, atol=1e-6, rtol=1e-5)
    assert torch.allclose(outs[1], emm, atol=1e-7, rtol=1e-5)
    assert torch.allclose(outs[2], ev, atol=1e-9, rtol=1e-4)
    assert torch.equal(pb, outs[0].to(torch.bfloat16))
    assert int(st[0]) == 0 and int(flag) == 0


def test_flag_wait_times_out_with_status_and_context_survives():
    dev = torch.device("cuda", 0)
    flags = ext().sym_alloc(64, 0).view(torch.int32)
    st = status_word(dev)
    st.zero_()
    # nothing ever sets this flag: the bounded wait must give up and report
    s1 = _step_block(dev, 1, 1e-3, 0.9, 0.999, 1)
    ext().flag_wait([flags[0].data_ptr()], s1, 0, st, 0.2)
    torch.cuda.synchronize()
    assert int(st[0]) == 2
    st.zero_()
    s7 = _step_block(dev, 7, 1e-3, 0.9, 0.999, 1)
    ext().flag_set(flags[0].data_ptr(), s7, 0)
    ext().flag_wait([flags[0].data_ptr()], s7, 0, st, 0.2)
    ext().flag_wait([flags[0].data_ptr()], s1, 6, st, 0.2)     # tag + delta
    torch.cuda.synchronize()
    assert int(st[0]) == 0 and int(flags[0]) == 7
    # K1 with an unset peer flag: records the timeout and writes nothing
    n = 4096
    master = torch.randn(n, device=dev)
    out = torch.full_like(master, 123.0)
    g = torch.randn(n, device=dev).to(torch.bfloat16)
    nf = torch.zeros(1, dtype=torch.int32, device=dev)
    s5 = _step_block(dev, 5, 1e-3, 0.9, 0.999, 1)
    ext().fused_reduce_adamw([g.data_ptr()], [flags[1].data_ptr()], s5, master, master, master, out, out.clone(),
                             out.clone(), torch.empty(n, device=dev, dtype=torch.bfloat16), 0.9, 0.999, 1e-8,
                             0.0, 1.0, nf, st, 0.2, 0)
    torch.cuda.synchronize()
    assert int(st[0]) == 2
    assert torch.all(out == 123.0)
    st.zero_()


def test_host_trip_ends_a_pending_peer_wait():
    """A peer seen dead on the host (PeerWatch.trip) ends a kernel that is
    already spinning on that peer's flag within one poll, not at its bound."""
    import time
    from shift_b200.ft.peer_watch import PeerWatch
    dev = torch.device("cuda", 0)
    flags = ext().sym_alloc(64, 0).view(torch.int32)
    st = status_word(dev)
    st.zero_()
    s1 = _step_block(dev, 1, 1e-3, 0.9, 0.999, 1)
    # built before the wait starts, as in training: its pinned source buffer is
    # allocated here (a pinned allocation can wait for the device to go idle)
    w = PeerWatch("me", st)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    ext().flag_wait([flags[0].data_ptr()], s1, 0, st, 10.0)     # nothing sets this flag; 10 s bound
    b.record()
    time.sleep(0.05)
    w.trip()
    torch.cuda.synchronize()
    w.close()
    assert int(st[0]) == 2
    assert a.elapsed_time(b) < 2000.0
    st.zero_()


def test_peer_copy_local():
    a = torch.randn(1 << 20, device="cuda")
    b = torch.empty_like(a)
    ext().peer_copy(a.data_ptr(), b.data_ptr(), a.numel() * 4)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _k1_worker(rank, world, port, q, mode):
    import torch.distributed as dist
    from datetime import timedelta

    from shift_b200.engine import Engine, synthetic_batch
    from shift_b200.models.qwen_moe import MoEConfig
    from shift_b200.parallel.replicas import _order
    from shift_b200.parallel.symmetric import CrossReplicaFused, SymmetricHeap
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=timedelta(seconds=60), device_id=dev)
    try:
        cfg = MoEConfig.tiny()
        B, S = 2, 128
        eng = Engine(cfg, dev, bucket_numel=1 << 18)
        heap = SymmetricHeap(dist.distributed_c10d._get_default_store(), f"r{rank}", dev)
        fused = CrossReplicaFused(eng, heap, timeout_s=20, mode=mode)
        dist.barrier()
        fused.configure([f"r{i}" for i in range(world)])
        eng.model.layer_done_hook = lambda layer: fused.on_layer_done(_order(layer, cfg.layers))
        for step in range(3):
            data = synthetic_batch(cfg, 100 * step + rank, B, S).to(dev)
            eng.nonfinite.zero_()
            fused.begin_step(step)
            eng.forward_backward([(data[:, :-1], data[:, 1:])], B, S)
            fused.finish_step()
            eng.commit()
        torch.cuda.synchronize()
        st = int(status_word(dev)[0])
        master = eng.store.state_tensors()["master"].cpu()
        if rank == 0:
            # single-process reference of the same three averaged steps
            r = Engine(cfg, dev, bucket_numel=1 << 18)
            grads = []
            for step in range(3):
                gl = []
                for src in range(world):
                    data = synthetic_batch(cfg, 100 * step + src, B, S).to(dev)
                    r.forward_backward([(data[:, :-1], data[:, 1:])], B, S)
                    gl.append(r.store.grad.clone())
                if mode == "two":
                    # the two-phase reduction averages in fp32 and rounds to bf16 before AdamW
                    avg = ((gl[0].float() + gl[1].float()) * (1.0 / world)).to(torch.bfloat16)
                    r.optimizer_step([avg], 1.0)
                else:
                    # one-phase: both bf16 gradients summed in fp32 inside the AdamW kernel, no rounding
                    r.optimizer_step([gl[0], gl[1]], 1.0 / world)
                r.commit()
                grads.append(gl)
            q.put(("ref", r.store.state_tensors()["master"].cpu()))
        q.put((rank, master, st))
        dist.barrier()
        heap.close_peers()
    finally:
        dist.destroy_process_group()


@pytest.mark.multigpu
@pytest.mark.parametrize("mode", ["auto", "two"])
def test_fused_cross_replica_two_gpus_bit_identical_and_matches_reference(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_k1_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world + 1):
        item = q.get(timeout=300)
        got[item[0]] = item
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    m0, m1 = got[0][1], got[1][1]
    assert got[0][2] == 0 and got[1][2] == 0
    assert torch.equal(m0, m1), "replicas diverged"
    refm = got["ref"][1]
    err = (m0 - refm).abs().max().item()
    assert err <= 1e-6, f"max |fused - reference| = {err}"
