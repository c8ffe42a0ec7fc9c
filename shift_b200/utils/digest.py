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


# ---------------------------------------------------------------------------
# Two-level SHA-256 tree digest of a flat buffer, computed where it lives.
#
# sha256tree(t) = SHA-256( str((dtype, shape)) || D_0 || D_1 || ... ) where D_i is
# the SHA-256 of the i-th consecutive LEAF-byte piece of the tensor's bytes
# (the last piece may be shorter).  On a CUDA tensor the leaf digests come from
# the sha256_leaves kernel (one thread per leaf); on the host from hashlib --
# the same value either way, so a GPU-side audit can be checked on the CPU.
# ---------------------------------------------------------------------------
LEAF = 1 << 16
_CONSTS: dict = {}


def _iroot(n: int, k: int) -> int:
    """floor(n ** (1/k)) for a non-negative integer, exactly (Newton)."""
    if n < 2:
        return n
    x = 1 << ((n.bit_length() + k - 1) // k)
    while True:
        y = ((k - 1) * x + n // x ** (k - 1)) // k
        if y >= x:
            return x
        x = y


def sha256_constants() -> list:
    """The 64 round constants (first 32 bits of the fractional parts of the
    cube roots of the first 64 primes) then the 8 initial hash words (square
    roots of the first 8 primes), computed exactly as FIPS 180-4 defines them."""
    primes, n = [], 2
    while len(primes) < 64:
        if all(n % p for p in primes if p * p <= n):
            primes.append(n)
        n += 1
    k = [_iroot(p << 96, 3) & 0xFFFFFFFF for p in primes]
    h = [_iroot(p << 64, 2) & 0xFFFFFFFF for p in primes[:8]]
    return k + h


def _consts_on(device) -> torch.Tensor:
    t = _CONSTS.get(device)
    if t is None:
        vals = [v - (1 << 32) if v >= 1 << 31 else v for v in sha256_constants()]
        t = _CONSTS[device] = torch.tensor(vals, dtype=torch.int32, device=device)
    return t


def leaf_digests(t: torch.Tensor, leaf: int = LEAF) -> bytes:
    t = t.detach().contiguous()
    if t.is_cuda:
        from ..ops._ext import ext
        return ext().sha256_leaves(t.reshape(-1), leaf, _consts_on(t.device)).cpu().numpy().tobytes()
    raw = t.reshape(-1).view(torch.uint8).numpy().tobytes()
    return b"".join(hashlib.sha256(raw[i:i + leaf]).digest() for i in range(0, len(raw), leaf))


def sha256tree(t: torch.Tensor, leaf: int = LEAF) -> str:
    h = hashlib.sha256(str((str(t.dtype), tuple(t.shape))).encode())
    h.update(leaf_digests(t, leaf))
    return h.hexdigest()
