"""State digests and tree helpers used by every audit.

``digest`` is the snapshot hash of the reference (shift_min/train.py:31-52,
shift_full/train.py:37-57): SHA-256 over, for a tensor, ``str((dtype, shape))``
followed by its raw bytes; for a dict, its items in the order of
``(type name, str(key))`` with key then value; for a list or tuple, ``str(type)``
then each item; for anything else ``repr(value)`` and a NUL byte.  Keeping the
same definition keeps hashes comparable across the two frameworks' evidence.
"""
from __future__ import annotations

import hashlib

import torch


def _feed(h, v):
    if isinstance(v, torch.Tensor):
        t = v.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        t = t.contiguous()
        h.update(str((str(t.dtype), tuple(t.shape))).encode())
        h.update(t.reshape(-1).view(torch.uint8).numpy().tobytes())
    elif isinstance(v, dict):
        for key in sorted(v, key=lambda k: (type(k).__name__, str(k))):
            _feed(h, key)
            _feed(h, v[key])
    elif isinstance(v, (list, tuple)):
        h.update(str(type(v)).encode())
        for item in v:
            _feed(h, item)
    else:
        h.update(repr(v).encode() + b"\0")


def digest(value) -> str:
    h = hashlib.sha256()
    _feed(h, value)
    return h.hexdigest()


def tensor_count(value) -> int:
    if isinstance(value, torch.Tensor):
        return 1
    if isinstance(value, dict):
        return sum(tensor_count(v) for v in value.values())
    if isinstance(value, (list, tuple)):
        return sum(tensor_count(v) for v in value)
    return 0


def cpu_tree(value):
    """Detached CPU copies of every tensor leaf (containers rebuilt)."""
    if isinstance(value, torch.Tensor):
        return value.detach().cpu().clone()
    if isinstance(value, dict):
        return {k: cpu_tree(v) for k, v in value.items()}
    if isinstance(value, list):
        return [cpu_tree(v) for v in value]
    if isinstance(value, tuple):
        return tuple(cpu_tree(v) for v in value)
    return value


def tree_bytes(value) -> int:
    if isinstance(value, torch.Tensor):
        return value.numel() * value.element_size()
    if isinstance(value, dict):
        return sum(tree_bytes(v) for v in value.values())
    if isinstance(value, (list, tuple)):
        return sum(tree_bytes(v) for v in value)
    return 0
