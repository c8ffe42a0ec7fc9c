"""Packed state transport (wire format of the reference's PackedGPUTransport).

A state pytree is flattened; tensor leaves that live on the transport's device
are packed per dtype into one flat buffer each; everything else travels in
pickled metadata.  On the wire, per destination and in this order:

    tag 1   int64 [1]   length of the metadata
    tag 2   uint8 [n]   pickled {version, step, treespec, groups, leaves,
                                 tensor_count, cpu_tensor_bytes}
    tag 3+i             flat buffer of dtype group i (skipped when empty)

``groups`` = [{dtype, numel}], ``leaves`` = [{kind: value|cpu|cuda|packed,
group, offset, shape | value}].  The receiver validates the version, the step,
every offset and the CPU byte count, then rebuilds the tree with views into the
received buffers.  Same layout, limits (16 MiB metadata, 4 MiB small CPU
leaves) and checks as shift_full/transport.py:24-321, so a frame sent by one
framework is readable by the other.  On a CPU (gloo) transport, CPU tensor
leaves are packed like device leaves and tagged ``packed``.
"""
from __future__ import annotations

import math
import pickle
import time
from datetime import timedelta
from typing import Any, Callable, Optional

import torch
from torch.utils._pytree import tree_flatten, tree_unflatten

MAX_METADATA_BYTES = 16 * 1024 * 1024
MAX_CPU_TENSOR_BYTES = 4 * 1024 * 1024
VERSION = 1


def pack_state(state: object, step: int, device: torch.device):
    """Returns (metadata bytes, [flat group tensors], tensor_count, cpu_tensor_bytes)."""
    device = torch.device(device)
    leaves, spec = tree_flatten(state)
    group_of: dict[torch.dtype, int] = {}
    parts: list[list[torch.Tensor]] = []
    numels: list[int] = []
    meta: list[dict[str, Any]] = []
    cpu_bytes = 0
    count = 0
    packed_kind = "cuda" if device.type == "cuda" else "packed"
    for v in leaves:
        if not isinstance(v, torch.Tensor):
            meta.append({"kind": "value", "value": v})
            continue
        count += 1
        if v.layout != torch.strided:
            raise TypeError(f"cannot pack a {v.layout} tensor: the wire format carries dense strided tensors")
        if v.device.type == device.type:
            g = group_of.get(v.dtype)
            if g is None:
                g = len(parts)
                group_of[v.dtype] = g
                parts.append([])
                numels.append(0)
            flat = v.detach().reshape(-1)
            meta.append({"kind": packed_kind, "group": g, "offset": numels[g], "shape": tuple(v.shape)})
            parts[g].append(flat)
            numels[g] += flat.numel()
        elif v.device.type == "cpu":
            cpu_bytes += v.numel() * v.element_size()
            if cpu_bytes > MAX_CPU_TENSOR_BYTES:
                raise ValueError(f"host-resident tensors in the state exceed {MAX_CPU_TENSOR_BYTES} bytes of control data")
            meta.append({"kind": "cpu", "value": v.detach().contiguous().clone()})
        else:
            raise TypeError(f"cannot pack a tensor that lives on {v.device}")
    groups = [torch.cat(p, 0) for p in parts]   # independent contiguous snapshots
    wire = {"version": VERSION, "step": step, "treespec": spec,
            "groups": [{"dtype": parts[i][0].dtype, "numel": numels[i]} for i in range(len(parts))],
            "leaves": meta, "tensor_count": count, "cpu_tensor_bytes": cpu_bytes}
    blob = pickle.dumps(wire, protocol=pickle.HIGHEST_PROTOCOL)
    if len(blob) > MAX_METADATA_BYTES:
        raise ValueError(f"pickled state description needs {len(blob)} bytes, more than the {MAX_METADATA_BYTES} allowed")
    return blob, groups, count, cpu_bytes


def unpack_state(wire: dict, groups: list[torch.Tensor]):
    leaves = []
    for leaf in wire["leaves"]:
        if not isinstance(leaf, dict):
            raise ValueError("state description: a leaf entry is not a well-formed record")
        kind = leaf.get("kind")
        if kind in ("value", "cpu"):
            leaves.append(leaf.get("value"))
        elif kind in ("cuda", "packed"):
            g, off, shape = leaf.get("group"), leaf.get("offset"), leaf.get("shape")
            if (not isinstance(g, int) or g < 0 or g >= len(groups) or not isinstance(off, int) or off < 0
                    or not isinstance(shape, (tuple, list)) or any(not isinstance(d, int) or d < 0 for d in shape)):
                raise ValueError("state description: a device leaf has a bad group, offset or shape")
            n = math.prod(shape)
            if off + n > groups[g].numel():
                raise ValueError("state description: a device leaf runs past the end of its flat buffer")
            leaves.append(groups[g].narrow(0, off, n).view(tuple(shape)))
        else:
            raise ValueError(f"state description: leaf kind {kind!r} is not value, cpu or cuda")
    return tree_unflatten(leaves, wire["treespec"])


def validate_wire(wire, step: int):
    if not isinstance(wire, dict) or wire.get("version") != VERSION:
        raise ValueError("state description has an unknown wire version")
    if wire.get("step") != step:
        raise ValueError(f"received the state of step {wire.get('step')} while expecting step {step}")
    if not isinstance(wire.get("groups"), list) or not isinstance(wire.get("leaves"), list):
        raise ValueError("state description is missing required fields")
    cpu = 0
    for leaf in wire["leaves"]:
        if isinstance(leaf, dict) and leaf.get("kind") == "cpu":
            v = leaf.get("value")
            if not isinstance(v, torch.Tensor) or v.device.type != "cpu" or v.layout != torch.strided:
                raise ValueError("state description: a host tensor entry is malformed")
            cpu += v.numel() * v.element_size()
            if cpu > MAX_CPU_TENSOR_BYTES:
                raise ValueError(f"host-resident tensors in the state exceed {MAX_CPU_TENSOR_BYTES} bytes of control data")
    if cpu != wire.get("cpu_tensor_bytes"):
        raise ValueError("host tensor bytes differ from the declared total")
    for i, g in enumerate(wire["groups"]):
        if (not isinstance(g, dict) or not isinstance(g.get("dtype"), torch.dtype) or not isinstance(g.get("numel"), int)
                or g["numel"] < 0):
            raise ValueError(f"flat buffer #{i} has a bad dtype or length")


class PackedTransport:
    """Checkpoint transport over a (reconfigurable) process group."""

    def __init__(self, pg, device, timeout: timedelta = timedelta(seconds=60),
                 event: Optional[Callable[..., None]] = None):
        self._pg = pg
        self._device = torch.device(device)
        self._timeout = timeout
        self._event = event

    def metadata(self) -> str:
        return "<packed-gpu>" if self._device.type == "cuda" else "<packed-cpu>"

    def disallow_checkpoint(self):
        pass

    def shutdown(self, wait: bool = True):
        pass

    def _emit(self, kind, step, seconds, gpu_bytes, control_bytes, tensors, cpu_bytes):
        if self._event is not None:
            self._event(kind, step=step, seconds=seconds, gpu_bytes=gpu_bytes, control_bytes=control_bytes,
                        tensors=tensors, cpu_tensor_bytes=cpu_bytes)

    def _sync(self):
        if self._device.type == "cuda":
            torch.cuda.current_stream(self._device).synchronize()

    def send_checkpoint(self, dst_ranks: list, step: int, state_dict: object, timeout=None, packed=None):
        start = time.perf_counter()
        blob, groups, count, cpu_bytes = packed if packed is not None else pack_state(state_dict, step, self._device)
        length = torch.tensor([len(blob)], dtype=torch.int64, device=self._device)
        meta = torch.frombuffer(bytearray(blob), dtype=torch.uint8).to(self._device)
        works = []
        for dst in dst_ranks:
            works.append(self._pg.send([length], dst, tag=1))
            works.append(self._pg.send([meta], dst, tag=2))
            for i, flat in enumerate(groups):
                if flat.numel() > 0:
                    works.append(self._pg.send([flat], dst, tag=3 + i))
        for w in works:
            w.wait()
        self._sync()
        self._emit("transport_send", step, time.perf_counter() - start,
                   sum(t.numel() * t.element_size() for t in groups), len(blob) + 8, count, cpu_bytes)

    def recv_checkpoint(self, src_rank: int, metadata: str, step: int, timeout=None):
        start = time.perf_counter()
        length = torch.empty(1, dtype=torch.int64, device=self._device)
        self._pg.recv([length], src_rank, tag=1).wait()
        n = int(length.item())
        if n <= 0 or n > MAX_METADATA_BYTES:
            raise ValueError(f"peer announced a {n}-byte state description (allowed: 1..{MAX_METADATA_BYTES})")
        meta = torch.empty(n, dtype=torch.uint8, device=self._device)
        self._pg.recv([meta], src_rank, tag=2).wait()
        wire = pickle.loads(meta.cpu().numpy().tobytes())
        validate_wire(wire, step)
        groups, works = [], []
        for i, g in enumerate(wire["groups"]):
            flat = torch.empty(g["numel"], dtype=g["dtype"], device=self._device)
            groups.append(flat)
            if g["numel"] > 0:
                works.append(self._pg.recv([flat], src_rank, tag=3 + i))
        for w in works:
            w.wait()
        result = unpack_state(wire, groups)
        self._sync()
        self._emit("transport_recv", step, time.perf_counter() - start,
                   sum(t.numel() * t.element_size() for t in groups), n + 8,
                   int(wire.get("tensor_count", len(wire["leaves"]))), wire["cpu_tensor_bytes"])
        return result


class FrozenTransport(PackedTransport):
    """Packs a snapshot once (``freeze``) and serves later sends from it:
    the P2 pre-copy read window (shift_full/overlap_handoff.py:15-22)."""

    def freeze(self, payload, step: int):
        self.frozen = pack_state(payload, step, self._device)
        self.frozen_step = step
        if self._device.type == "cuda":
            self.ready = torch.cuda.Event()
            self.ready.record()
        else:
            self.ready = None

    def send_checkpoint(self, dst_ranks, step, state_dict, timeout=None, packed=None):
        if step != self.frozen_step:
            raise ValueError("a frozen tensor was modified while its snapshot was being sent")
        if self.ready is not None:
            self.ready.wait()
        return super().send_checkpoint(dst_ranks, step, None, timeout, packed=self.frozen)
