"""Symmetric peer memory over CUDA IPC, and the cross-replica fused optimizer.

``SymmetricHeap``: named, IPC-exportable allocations per rank; handles are
published in a ``torch.distributed`` store under ``sym/<owner>/<name>`` and
peers map them once (re-mapping for a new membership is a store lookup plus
``cudaIpcOpenMemHandle``, not a communicator rebuild).

``CrossReplicaFused``: the K1 path.  Each rank keeps two IPC-exported bf16
gradient buffers (alternating by step, so a peer can still be reading step
s-1 while this rank writes step s) and a flag block
``[ready[n_buckets], done[2]]``.  During backward, when a bucket's last layer
has written its gradient, the rank publishes ``ready[b] = tag(step)`` on the
compute stream and launches the fused reduce + AdamW for that bucket on a
side stream; the kernel waits (bounded) for every participant's
``ready[b]``, reads their gradients over NVLink in replica order, and writes
the next state generation.  After the last bucket the rank publishes
``done[parity]``; the next use of that gradient buffer first waits for
every peer's ``done`` of two steps back.  All waits are bounded and report
through the kernel status word.
"""
from __future__ import annotations

import os

import torch

from ..ops._ext import ext, status_word


class SymmetricHeap:
    def __init__(self, store, owner: str, device: torch.device):
        self.store = store
        self.owner = owner
        self.device = torch.device(device)
        self.local: dict[str, torch.Tensor] = {}
        self.peers: dict[tuple, torch.Tensor] = {}

    def alloc(self, name: str, nbytes: int) -> torch.Tensor:
        t = ext().sym_alloc(int(nbytes), self.device.index)
        self.local[name] = t
        h = ext().ipc_handle(t)
        self.handles = getattr(self, "handles", {})
        self.handles[name] = bytes(h.numpy().tobytes()) + int(nbytes).to_bytes(8, "little")
        if self.store is not None:
            self.store.set(f"sym/{self.owner}/{name}", self.handles[name])
        return t

    def publish(self, store, make_default: bool = True):
        """(Re)publish every local handle into ``store`` (e.g. a new quorum's store)."""
        if make_default:
            self.store = store
        for name, blob in getattr(self, "handles", {}).items():
            store.set(f"sym/{self.owner}/{name}", blob)

    def open(self, owner: str, name: str, store=None) -> torch.Tensor:
        key = (owner, name)
        if owner == self.owner:
            return self.local[name]
        t = self.peers.get(key)
        if t is None:
            raw = (store or self.store).get(f"sym/{owner}/{name}")
            h = torch.frombuffer(bytearray(raw[:64]), dtype=torch.uint8)
            nbytes = int.from_bytes(raw[64:72], "little")
            t = ext().ipc_open(h, nbytes, self.device.index)
            self.peers[key] = t
        return t

    def close_peers(self):
        self.peers.clear()


def _tag(step: int) -> int:
    return step + 1


class CrossReplicaFused:
    """K1 for one rank: fused cross-replica gradient reduction + AdamW."""

    def __init__(self, engine, heap: SymmetricHeap, timeout_s: float = 30.0, two_phase: bool = True,
                 mode: str | None = None):
        self.engine = engine
        self.heap = heap
        self.timeout = timeout_s
        st = engine.store
        self.numel = st.numel
        nbytes = self.numel * 2
        self.gbuf = [heap.alloc(f"grad{i}", nbytes).view(torch.bfloat16)[: self.numel] for i in range(2)]
        self.nb = len(st.buckets)
        # flags: ready[nb] | done[2] | slice[nb]
        self.flags = heap.alloc("flags", 4 * (2 * self.nb + 2) + 64).view(torch.int32)
        # K1 form per segment: "auto" reads every source directly and sums in
        # fp32 when a segment has at most two sources (one peer: the same NVLink
        # bytes per direction as reduce-scatter + all-gather, and no bf16
        # rounding of the sum), and uses the two-phase slice form above that;
        # "one" / "two" force a form; "nccl" is the baseline: NCCL all_reduce
        # of each bucket on the side stream, then the local fused AdamW.
        self.mode = mode or os.environ.get("SHIFT_K1", "auto")
        if self.mode not in ("auto", "one", "two", "nccl"):
            raise ValueError(f"SHIFT_K1={self.mode!r}: expected auto, one, two or nccl")
        self.nccl_group = None
        # reduced gradient written by every member's slice (two-phase K1)
        self.two_phase = two_phase and self.mode != "one"
        if two_phase:
            self.red = heap.alloc("red", nbytes).view(torch.bfloat16)[: self.numel]
        st.set_grad_buffers(self.gbuf)
        self.side = torch.cuda.Stream(device=heap.device)
        self.peer_owners: list[str] = [heap.owner]
        self.scale = 1.0
        self.status = status_word(heap.device)
        # bucket completion order (backward order: head, layers high->low, embed)
        layers = engine.cfg.layers
        order_of = {}
        for s in st.specs:
            if s.layer >= 0:
                order_of[s.name] = layers - s.layer
            elif s.name.startswith("embed"):
                order_of[s.name] = layers + 1
            else:
                order_of[s.name] = 0
        self.bucket_done_at = [max(order_of[n] for n in b.names) for b in st.buckets]
        self.step = 0
        self.launched: set[int] = set()
        self.active = False
        # blocks per SM of the launches during backward (0 = the whole GPU).  One
        # block per SM lets the reduction co-reside with the compute kernels,
        # but measured slower on two B200s (24.5 vs 21.9 ms per step): the
        # stretched reduction competes for HBM with the memory-bound parts of
        # backward for longer than the short full-GPU bursts stall it
        self.overlap_blocks_per_sm = int(os.environ.get("SHIFT_K1_OVERLAP_BLOCKS", "0"))

    # ------------------------------------------------------------------ membership
    def configure(self, owners_in_replica_order: list[str], participating: list[bool] | None = None,
                  step: int = 0):
        """owners of the same shard in every replica of the quorum (replica order).
        ``participating[i]`` False -> that replica contributes zeros (healing/spare).
        ``step``: the step this membership starts at (peers that joined later
        than two steps ago are not waited on for buffer reuse)."""
        self.peer_owners = list(owners_in_replica_order)
        part = participating or [True] * len(owners_in_replica_order)
        self.sources = [o for o, p in zip(self.peer_owners, part) if p]
        if not 1 <= len(self.sources) <= 8:
            raise ValueError("1..8 participating replicas supported by the fused path")
        self.scale = 1.0 / len(self.sources)
        since = getattr(self, "member_since", {})
        self.member_since = {o: since.get(o, step) for o in self.peer_owners}
        self.grad_maps = {o: [self.heap.open(o, f"grad{i}").view(torch.bfloat16)[: self.numel] for i in range(2)]
                          for o in self.peer_owners}
        self.flag_maps = {o: self.heap.open(o, "flags").view(torch.int32) for o in self.peer_owners}
        if self.two_phase:
            self.red_maps = {o: self.heap.open(o, "red").view(torch.bfloat16)[: self.numel] for o in self.peer_owners}
        self.segments = [(0, self.numel, self.sources, self.scale, list(self.peer_owners))]

    def configure_segments(self, owners: list[str], segments: list, step: int = 0):
        """Different flat ranges reduced over different source sets.
        segments: [(lo, hi, source_owners_in_fixed_order, scale)].  With tensor
        parallelism the TP-replicated parameters are summed over the TP pair
        and averaged over replicas, the TP-sharded ones only averaged over
        replicas."""
        self.configure(owners, None, step)
        for lo, hi, srcs, _ in segments:
            if not 1 <= len(srcs) <= 8:
                raise ValueError("1..8 gradient sources per segment")
            for o in srcs:
                if o not in self.peer_owners:
                    raise ValueError(f"segment source {o} is not a member")
        self.segments = list(segments)

    # ------------------------------------------------------------------ per step
    def begin_step(self, step: int, defer: bool = False, prepare: bool = True):
        """Select this step's gradient buffer; make sure every peer finished
        reading it two steps ago.  ``defer``: launch no bucket during backward
        (membership may change before the reduction, e.g. a gradient relay);
        ``finish_step`` then launches every bucket.  ``prepare=False``: the
        caller already wrote the engine's step block (``prepare_step(tag)``),
        as it must when this step is being captured into a CUDA graph."""
        self.step = step
        par = step % 2
        self.engine.store.select_grad(par)
        if prepare:
            self.engine.prepare_step(_tag(step))
        self.sdev = self.engine.step_block.dev
        if step >= 2:
            since = getattr(self, "member_since", {})
            ptrs = [self.flag_maps[o][self.nb + par].data_ptr() for o in self.peer_owners
                    if o != self.heap.owner and since.get(o, 0) <= step - 2]
            ext().flag_wait(ptrs, self.sdev, -2, self.status, self.timeout)
        self.launched = set()
        self.active = not defer
        self.progress = -1

    def on_layer_done(self, order: int):
        """Called from the model's backward (last microbatch) as layers finish."""
        if not self.active:
            return
        self.progress = max(self.progress, order)
        for b in range(self.nb):
            if b not in self.launched and self.bucket_done_at[b] <= self.progress:
                self._launch(b)

    def _launch(self, b: int):
        st = self.engine.store
        bk = st.buckets[b]
        par = self.step % 2
        tag = _tag(self.step)
        my_flags = self.flags
        ext().flag_set(my_flags[b].data_ptr(), self.sdev, 0)   # compute stream: grads of bucket b are written
        ev = torch.cuda.Event()
        ev.record()
        with torch.cuda.stream(self.side):
            self.side.wait_event(ev)
            c, n = st.cur, st.nxt
            o = self.engine.optim
            if self.mode == "nccl":
                self._nccl(b, bk, c, n, o)
                self.launched.add(b)
                return
            if self.two_phase:
                self._two_phase(b, bk, par, tag, c, n, o)
            for seg in self.segments:
                lo, hi, srcs, scale = seg[:4]
                s0, s1 = max(bk.start, lo), min(bk.end, hi)
                if s0 >= s1 or self._sliced(srcs):
                    continue
                sl = slice(s0, s1)
                grad_ptrs = [self.grad_maps[w][par][sl].data_ptr() for w in srcs]
                flag_ptrs = [self.flag_maps[w][b].data_ptr() for w in srcs if w != self.heap.owner]
                ext().fused_reduce_adamw(grad_ptrs, flag_ptrs, self.sdev, st.master[c][sl], st.exp_avg[c][sl],
                                         st.exp_avg_sq[c][sl], st.master[n][sl], st.exp_avg[n][sl],
                                         st.exp_avg_sq[n][sl], st.param[n][sl], o.beta1, o.beta2, o.eps,
                                         o.weight_decay, scale, self.engine.nonfinite, self.status, self.timeout,
                                         self._grid())
        self.launched.add(b)

    def _grid(self) -> int:
        """Blocks per SM of a reduction launch: ``overlap_blocks_per_sm`` while
        backward is still running, the whole GPU for buckets launched after
        backward."""
        return self.overlap_blocks_per_sm if self.active else 0

    def _sliced(self, srcs) -> bool:
        """Whether a segment with these sources takes the two-phase form."""
        return self.two_phase and (self.mode == "two" or len(srcs) > 2)

    def _nccl(self, b, bk, c, n, o):
        """Baseline K1: NCCL all_reduce (sum) of the bucket's bf16 gradient over
        the replicas, then AdamW with the 1/R scale from the local buffer."""
        import torch.distributed as dist
        st = self.engine.store
        if self.nccl_group is None:
            raise RuntimeError("SHIFT_K1=nccl needs nccl_group (the replicas' process group)")
        sl = slice(bk.start, bk.end)
        g = st.grad[sl]
        dist.all_reduce(g, group=self.nccl_group)
        ext().fused_reduce_adamw([g.data_ptr()], [], self.sdev, st.master[c][sl], st.exp_avg[c][sl],
                                 st.exp_avg_sq[c][sl], st.master[n][sl], st.exp_avg[n][sl], st.exp_avg_sq[n][sl],
                                 st.param[n][sl], o.beta1, o.beta2, o.eps, o.weight_decay, self.scale,
                                 self.engine.nonfinite, self.status, self.timeout, self._grid())

    def _two_phase(self, b, bk, par, tag, c, n, o):
        """Phase A: reduce this rank's slice of every segment and store it into
        every member's reduced buffer; publish slice[b].  Phase B: AdamW from
        the local reduced gradient once every source's slice has landed."""
        st = self.engine.store
        me = self.heap.owner
        slice_flag = self.nb + 2 + b
        parts = []
        for seg in self.segments:
            lo, hi, srcs, scale = seg[:4]
            # receivers: the sources plus, for the whole-model segment of a
            # quorum, members that do not contribute (healing / spare)
            members = seg[4] if len(seg) > 4 else list(srcs)
            s0, s1 = max(bk.start, lo), min(bk.end, hi)
            if s0 >= s1 or not self._sliced(srcs):
                continue
            parts.append((s0, s1, srcs))
            if me not in srcs:
                continue           # a non-participating member only receives
            k, ns = srcs.index(me), len(srcs)
            cuts = [s0 + ((s1 - s0) * j // ns) // 8 * 8 for j in range(ns)] + [s1]
            ext().reduce_slice_scatter([self.grad_maps[w][par].data_ptr() for w in srcs],
                                       [self.red_maps[w].data_ptr() for w in members], cuts[k], cuts[k + 1],
                                       [self.flag_maps[w][b].data_ptr() for w in srcs if w != me], self.sdev,
                                       scale, self.status, self.timeout, self._grid())
        if not parts:
            return
        ext().flag_set(self.flags[slice_flag].data_ptr(), self.sdev, 0)
        for s0, s1, srcs in parts:
            sl = slice(s0, s1)
            ext().fused_reduce_adamw([self.red[sl].data_ptr()],
                                     [self.flag_maps[w][slice_flag].data_ptr() for w in srcs if w != me], self.sdev,
                                     st.master[c][sl], st.exp_avg[c][sl], st.exp_avg_sq[c][sl], st.master[n][sl],
                                     st.exp_avg[n][sl], st.exp_avg_sq[n][sl], st.param[n][sl], o.beta1, o.beta2,
                                     o.eps, o.weight_decay, 1.0, self.engine.nonfinite, self.status, self.timeout,
                                     self._grid())

    def finish_step(self):
        """After backward: launch what is left, publish done, join streams."""
        self.active = False          # nothing left to overlap with: full-GPU launches
        for b in range(self.nb):
            if b not in self.launched:
                self._launch(b)
        cur = torch.cuda.current_stream()
        cur.wait_stream(self.side)
        ext().flag_set(self.flags[self.nb + self.step % 2].data_ptr(), self.sdev, 0)
        self.active = False
        return self.engine.nonfinite
