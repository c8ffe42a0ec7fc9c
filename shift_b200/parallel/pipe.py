"""Pipeline-parallel send / receive between adjacent stages of one replica.

The 1F1B schedule (``parallel.tp_pp``) moves two things per microbatch: the
stage output (residual stream ``h`` and the pending MoE delta, [2, T, H] bf16)
forward, and the gradient w.r.t. the stage input ([T, H]; both halves of the
pair receive the same gradient) backward.  The reference runs these on NCCL
p2p inside Megatron's 1F1B (shift_full/train.py:552-554).

``PipePeer`` (default) moves them over NVLink peer memory: the sender's
``xcopy`` kernel stores the tensor straight into the receiver's buffer for
that (step parity, microbatch) and, after a system-scope fence, publishes its
own flag = step tag; the receiver's first consumer is preceded by a bounded
in-kernel wait on that flag.  Sends never block the sender's stream, receives
are a single-CTA wait on the compute stream, buffers are allocated once, and
the whole step -- pipeline exchanges included -- is a CUDA graph.  Buffer
reuse is safe without extra handshakes: a buffer of parity p is rewritten two
steps later, and 1F1B's data dependencies already order that write after the
receiver's last read (a stage starts step s+1 only after receiving the last
gradient of step s, which its neighbour sends after consuming all of step s's
activations).

``PipeNccl`` is the NCCL baseline: batched ``isend``/``irecv`` pairs into
receive buffers allocated once (matched pairs avoid the deadlock of two
blocking sends crossing), waited on by the compute stream only.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

ACT, GRAD = "act", "grad"


class PipeNccl:
    name = "nccl"
    graphable = False

    def __init__(self, group, ranks: list, stage: int, act_shape, grad_shape, microbatches: int, device):
        self.group, self.ranks, self.s = group, ranks, stage
        self.bufs = {}
        for i in range(microbatches):
            if stage > 0:
                self.bufs[(ACT, i)] = torch.empty(act_shape, dtype=torch.bfloat16, device=device)
            if stage < len(ranks) - 1:
                self.bufs[(GRAD, i)] = torch.empty(grad_shape, dtype=torch.bfloat16, device=device)

    def set_parity(self, parity: int):
        pass

    def exchange(self, send=None, recv=None):
        """send = (kind, microbatch, tensor); recv = (kind, microbatch).
        Activations go to stage s+1 and come from s-1; gradients the reverse."""
        ops, buf = [], None
        if send is not None:
            kind, _, t = send
            dst = self.s + 1 if kind == ACT else self.s - 1
            ops.append(dist.P2POp(dist.isend, t.contiguous(), self.ranks[dst], group=self.group))
        if recv is not None:
            kind, i = recv
            src = self.s - 1 if kind == ACT else self.s + 1
            buf = self.bufs[(kind, i)]
            ops.append(dist.P2POp(dist.irecv, buf, self.ranks[src], group=self.group))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()          # orders the compute stream after the transfer; the host does not block
        return buf


class PipePeer:
    name = "peer"
    graphable = True

    def __init__(self, heap, owners: list, stage: int, act_shape, grad_shape, microbatches: int, device,
                 sdev: torch.Tensor, timeout_s: float = 30.0):
        from ..ops._ext import status_word
        self.heap, self.owners, self.s = heap, owners, stage
        self.M = microbatches
        self.act_shape, self.grad_shape = tuple(act_shape), tuple(grad_shape)
        self.act_numel = _numel(act_shape)
        self.grad_numel = _numel(grad_shape)
        # receive slots of this rank: act[par][i] (from s-1), grad[par][i] (from s+1)
        self.slots, nbytes = _slots(stage, len(owners), microbatches, self.act_numel, self.grad_numel)
        self.arena = heap.alloc("pp_arena", max(nbytes, 256)).view(torch.bfloat16)
        # flags this rank publishes: sent_act[i], sent_grad[i]; one CTA counter per flag after them
        self.nflags = 2 * microbatches
        self.flags = heap.alloc("pp_flags", 8 * self.nflags + 64).view(torch.int32)
        self.sdev = sdev
        self.status = status_word(torch.device(device))
        self.timeout = timeout_s
        self.par = 0
        self.peer_arena, self.peer_flags, self.peer_slots = {}, {}, {}

    def connect(self):
        """Map the neighbours' arenas and flags (after every rank allocated them)."""
        for nb in (self.s - 1, self.s + 1):
            if 0 <= nb < len(self.owners):
                self.peer_arena[nb] = self.heap.open(self.owners[nb], "pp_arena").view(torch.bfloat16)
                self.peer_flags[nb] = self.heap.open(self.owners[nb], "pp_flags").view(torch.int32)
                self.peer_slots[nb] = _slots(nb, len(self.owners), self.M, self.act_numel, self.grad_numel)[0]

    def set_parity(self, parity: int):
        self.par = parity

    def _flag_index(self, kind, i):
        return (0 if kind == ACT else self.M) + i

    def _view(self, arena, slots, kind, i):
        off = slots[(kind, self.par, i)]
        n = self.act_numel if kind == ACT else self.grad_numel
        shape = self.act_shape if kind == ACT else self.grad_shape
        return arena[off // 2: off // 2 + n].view(shape)

    def send(self, kind, i, t: torch.Tensor):
        """Store ``t`` into the neighbour's slot, then publish our flag."""
        from ..ops._ext import ext
        nb = self.s + 1 if kind == ACT else self.s - 1
        dst = self._view(self.peer_arena[nb], self.peer_slots[nb], kind, i)
        t = t.contiguous()
        if t.numel() != dst.numel() or t.dtype != torch.bfloat16:
            raise ValueError(f"pipeline {kind}: {t.numel()} {t.dtype} elements for a bf16 slot of {dst.numel()}")
        j = self._flag_index(kind, i)
        xc = [0, 0, self.flags[j].data_ptr(), self.flags[self.nflags + j].data_ptr(), 0, self.sdev.data_ptr(),
              dst.data_ptr()]
        ext().xcopy(t.data_ptr(), 0, t.numel() * 2, xc, self.status)

    def recv(self, kind, i) -> torch.Tensor:
        """Bounded in-stream wait for the neighbour's flag; returns our slot."""
        from ..ops._ext import ext
        nb = self.s - 1 if kind == ACT else self.s + 1
        j = self._flag_index(kind, i)
        ext().flag_wait([self.peer_flags[nb][j].data_ptr()], self.sdev, 0, self.status, self.timeout)
        return self._view(self.arena, self.slots, kind, i)

    def exchange(self, send=None, recv=None):
        if send is not None:
            self.send(*send)
        return None if recv is None else self.recv(*recv)


def _numel(shape) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def _slots(stage: int, n_stages: int, microbatches: int, act_numel: int, grad_numel: int):
    """Byte offsets of a stage's receive slots, keyed (kind, parity,
    microbatch), each rounded up to 256 bytes; and the arena size."""
    slots, off = {}, 0
    for par in (0, 1):
        for i in range(microbatches):
            if stage > 0:
                slots[(ACT, par, i)] = off
                off += -(-act_numel * 2 // 256) * 256
            if stage < n_stages - 1:
                slots[(GRAD, par, i)] = off
                off += -(-grad_numel * 2 // 256) * 256
    return slots, off
