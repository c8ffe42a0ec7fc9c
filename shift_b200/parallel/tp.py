"""Tensor parallelism with sequence parallelism over a pair of GPUs.

The residual stream is split along tokens: TP rank r holds tokens
[r*T/tp, (r+1)*T/tp) of every microbatch.  Column-parallel projections
(QKV, and the expert block, whose experts are split over the pair: EP = TP,
ETP = 1) consume the all-gathered activation; row-parallel projections
(attention output, expert combine) produce partial sums that are
reduce-scattered back to the token split.  In backward, all-gather and
reduce-scatter swap roles.  This is Megatron's TP + SP with EP laid over the
TP group -- the layout the reference runs inside each replica
(shift_full/train.py:201-216, sequence_parallel off there), on one box.

``TPComm`` implements the two collectives.  ``backend="nccl"`` uses the TP
process group; ``backend="peer"`` uses symmetric peer buffers and the
peer-memory kernels (gathered halves are written straight into the peer's
buffer; reduce-scatter adds the peer's partial half in a fixed rank order).
"""
from __future__ import annotations

import threading

import torch
import torch.distributed as dist


class TPComm:
    def __init__(self, group, rank: int, size: int, device):
        self.group = group
        self.rank = rank
        self.size = size
        self.device = torch.device(device)

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        """[T/tp, H] -> [T, H] (rank order)."""
        if self.size == 1:
            return x
        out = torch.empty((x.shape[0] * self.size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def reduce_scatter(self, x: torch.Tensor) -> torch.Tensor:
        """[T, H] partial sums -> [T/tp, H] of the sum."""
        if self.size == 1:
            return x
        out = torch.empty((x.shape[0] // self.size,) + tuple(x.shape[1:]), dtype=x.dtype, device=x.device)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
        return out

    def all_reduce_(self, x: torch.Tensor) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(x, group=self.group)
        return x

    def local_rows(self, x: torch.Tensor) -> torch.Tensor:
        n = x.shape[0] // self.size
        return x[self.rank * n:(self.rank + 1) * n]


_CPU_PEERS: dict = {}


class CpuXchg:
    """Host stand-in for the kernels' exchange hooks (two ranks as threads):
    ``before`` waits for the peer's event, ``after`` sets ours; ``peer_out``
    is the peer's destination tensor."""

    def __init__(self, wait_ev=None, sig_ev=None, peer_out=None, timeout_s: float = 60.0):
        self.wait_ev, self.sig_ev, self.peer_out, self.timeout = wait_ev, sig_ev, peer_out, timeout_s

    def before(self):
        if self.wait_ev is not None and not self.wait_ev.wait(self.timeout):
            raise TimeoutError("tensor-parallel peer never signalled")

    def after(self):
        if self.sig_ev is not None:
            self.sig_ev.set()


_FULL = ("gA", "gM", "gD", "gH")      # gathered [T, H]: ln1 out, ln2 out, layer-output grad, ln2-input grad
_HALF = ("rAttn", "rMoe", "rDm", "rDa")  # received partial sums [T/2, H] of this rank's rows


class TPPeer(TPComm):
    """Tensor-parallel pair over symmetric peer memory: no collective library
    on the activation path.

    Every exchange point of a layer has a buffer in a per-rank arena that
    both ranks map (CUDA IPC), for each layer of the stage, microbatch slot
    and step parity (a buffer is rewritten two steps later, after the
    cross-replica reduction of the step in between has synchronised every
    member), and a flag + CTA counter.

    * all-gather (``_FULL`` kinds): the kernel that produces this rank's
      rows (RMSNorm forward / backward, or ``xcopy``) writes them into its
      own gather buffer AND into the peer's, then signals; the consumer (a
      GEMM) waits in-kernel for the peer's flag before its first TMA load of
      the peer's rows, starting on its own rows (rotated tile order).
    * reduce-scatter (``_HALF`` kinds): the kernel that produces the partial
      sums (GEMM epilogue, MoE combine, router input-gradient) stores the
      peer's rows into the peer's receive buffer and signals; the consuming
      RMSNorm waits for the flag and adds both partials in fp32.

    A flag holds the step tag of the last completed write (from the device
    step block), so graphs replay without host involvement; every wait is
    bounded and reports through the status word.  The collective semantics
    are those of Megatron TP + SP with EP over the TP pair (all-gather in
    rank order; reduce-scatter of row halves).
    """

    fused = True

    def __init__(self, group, rank: int, size: int, device, heap, peer_owner: str, tokens: int, hidden: int,
                 layers, microbatches: int, timeout_s: float = 30.0):
        super().__init__(group, rank, size, device)
        if size != 2:
            raise ValueError("TPPeer pairs exactly two ranks")
        if tokens % 256:
            raise ValueError("tokens per microbatch must be a multiple of 256 (two 128-row halves)")
        from ..ops._ext import status_word
        self.heap, self.peer_owner = heap, peer_owner
        self.T, self.H, self.half = tokens, hidden, tokens // 2
        self.layers = list(layers)
        self.M = microbatches
        self.index = {}
        off = 0
        for par in (0, 1):
            for mb in range(microbatches):
                for layer in self.layers:
                    for kind in _FULL + _HALF:
                        rows = tokens if kind in _FULL else self.half
                        self.index[(kind, layer, mb, par)] = (off, rows)
                        off += -(-rows * hidden * 2 // 256) * 256
        self.nbytes = off
        self.flag_of = {}
        for mb in range(microbatches):
            for layer in self.layers:
                for kind in _FULL + _HALF:
                    self.flag_of[(kind, layer, mb)] = len(self.flag_of)
        self.nflags = len(self.flag_of)
        self.cpu = self.device.type != "cuda"
        if self.cpu:
            # two ranks as two threads of one process (host-logic tests): the
            # "peer memory" is the other thread's arena, flags are events
            self.arena = torch.zeros(self.nbytes // 2, dtype=torch.float32)
            self.events = [threading.Event() for _ in range(self.nflags)]
            _CPU_PEERS[heap.owner] = self
            self.status = None
        else:
            self.arena = heap.alloc("tp_arena", self.nbytes).view(torch.bfloat16)
            self.flags = heap.alloc("tp_flags", 8 * self.nflags + 64).view(torch.int32)
            self.status = status_word(self.device)
        self.timeout = timeout_s
        self.par = 0
        self.mb = 0
        self.sdev = None

    def connect(self, sdev: torch.Tensor):
        """Map the peer's arena and flags (after both ranks allocated them)."""
        self.sdev = sdev
        if self.cpu:
            self.peer = _CPU_PEERS[self.peer_owner]
            self.peer_arena = self.peer.arena
            return
        self.peer_arena = self.heap.open(self.peer_owner, "tp_arena").view(torch.bfloat16)
        self.peer_flags = self.heap.open(self.peer_owner, "tp_flags").view(torch.int32)

    # ------------------------------------------------------------------ slots
    def set_slot(self, microbatch: int, parity: int):
        self.mb, self.par = microbatch, parity

    def _view(self, arena, kind, layer):
        off, rows = self.index[(kind, layer, self.mb, self.par)]
        return arena[off // 2: off // 2 + rows * self.H].view(rows, self.H)

    def reset_flags(self):
        """CPU emulation only: forget completed exchanges before the next step."""
        for e in self.events:
            e.clear()

    def buf(self, kind: str, layer: int) -> torch.Tensor:
        return self._view(self.arena, kind, layer)

    def pbuf(self, kind: str, layer: int) -> torch.Tensor:
        return self._view(self.peer_arena, kind, layer)

    def own(self) -> slice:
        return slice(self.rank * self.half, (self.rank + 1) * self.half)

    def peer_range(self) -> tuple[int, int]:
        p = 1 - self.rank
        return p * self.half, (p + 1) * self.half

    def rot_own_first(self) -> int:
        """Row-tile rotation that starts a GEMM on this rank's rows."""
        return (self.rank * self.half) // 128

    def rot_peer_first(self) -> int:
        return ((1 - self.rank) * self.half) // 128

    # ------------------------------------------------------------------ exchange args
    def _flag(self, flags, kind, layer):
        j = self.flag_of[(kind, layer, self.mb)]
        return flags[j].data_ptr(), flags[self.nflags + j].data_ptr()

    def xchg(self, wait=None, sig=None, peer_out: torch.Tensor | None = None):
        """[wait_flag, wait_delta, sig_flag, sig_counter, sig_delta, sdev, peer_out] for the kernels.
        wait=(kind, layer): the peer's flag of that exchange; sig=(kind, layer): ours.
        On CPU: a CpuXchg the reference implementations of the ops honour."""
        if self.cpu:
            j = lambda ks: self.flag_of[(ks[0], ks[1], self.mb)]
            return CpuXchg(None if wait is None else self.peer.events[j(wait)],
                           None if sig is None else self.events[j(sig)], peer_out)
        wf = self._flag(self.peer_flags, *wait)[0] if wait is not None else 0
        sf, sc = self._flag(self.flags, *sig) if sig is not None else (0, 0)
        po = peer_out.data_ptr() if peer_out is not None else 0
        return [wf, 0, sf, 0 if sig is None else sc, 0, self.sdev.data_ptr(), po]

    def wait(self, kind: str, layer: int):
        """A stand-alone bounded wait on the peer's flag (for consumers that
        are not exchange-aware kernels)."""
        if self.cpu:
            self.xchg(wait=(kind, layer)).before()
            return
        from ..ops._ext import ext
        ext().flag_wait([self._flag(self.peer_flags, kind, layer)[0]], self.sdev, 0, self.status, self.timeout)

    def push(self, src: torch.Tensor, kind: str, layer: int):
        """Copy this rank's rows into its own and the peer's gather buffer of
        (kind, layer), then signal (the producer was not an exchange-aware kernel)."""
        from ..ops._ext import ext
        own = self.own()
        dst, pdst = self.buf(kind, layer)[own], self.pbuf(kind, layer)[own]
        src = src.contiguous()
        if self.cpu:
            dst.copy_(src)
            pdst.copy_(src)
            self.xchg(sig=(kind, layer)).after()
            return
        ext().xcopy(src.data_ptr(), dst.data_ptr(), src.numel() * src.element_size(),
                    self.xchg(sig=(kind, layer), peer_out=pdst), self.status)
