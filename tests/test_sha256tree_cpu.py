"""The tree digest's building blocks on the host: the SHA-256 constants
computed from the primes drive a plain restatement of the compression
function that reproduces hashlib, and the host tree digest is the SHA-256 of
the leaf digests."""
import hashlib
import struct

import torch

from shift_b200.utils.digest import LEAF, leaf_digests, sha256_constants, sha256tree


def _sha256(msg: bytes, consts) -> bytes:
    k, h = consts[:64], list(consts[64:])
    m = msg + b"\x80" + b"\0" * ((55 - len(msg)) % 64) + struct.pack(">Q", 8 * len(msg))
    r = lambda x, n: ((x >> n) | (x << (32 - n))) & 0xFFFFFFFF  # noqa: E731
    for off in range(0, len(m), 64):
        w = list(struct.unpack(">16I", m[off:off + 64]))
        for t in range(16, 64):
            s0 = r(w[t - 15], 7) ^ r(w[t - 15], 18) ^ (w[t - 15] >> 3)
            s1 = r(w[t - 2], 17) ^ r(w[t - 2], 19) ^ (w[t - 2] >> 10)
            w.append((w[t - 16] + s0 + w[t - 7] + s1) & 0xFFFFFFFF)
        a, b, c, d, e, f, g, hh = h
        for t in range(64):
            t1 = (hh + (r(e, 6) ^ r(e, 11) ^ r(e, 25)) + ((e & f) ^ (~e & g)) + k[t] + w[t]) & 0xFFFFFFFF
            t2 = ((r(a, 2) ^ r(a, 13) ^ r(a, 22)) + ((a & b) ^ (a & c) ^ (b & c))) & 0xFFFFFFFF
            a, b, c, d, e, f, g, hh = (t1 + t2) & 0xFFFFFFFF, a, b, c, (d + t1) & 0xFFFFFFFF, e, f, g
        h = [(x + y) & 0xFFFFFFFF for x, y in zip(h, (a, b, c, d, e, f, g, hh))]
    return struct.pack(">8I", *h)


def test_constants_reproduce_hashlib():
    consts = sha256_constants()
    assert len(consts) == 72
    for msg in (b"", b"abc", bytes(range(55)), bytes(range(56)), bytes(range(64)), bytes(range(200)) * 3):
        assert _sha256(msg, consts) == hashlib.sha256(msg).digest()


def test_host_tree_digest():
    t = torch.arange(3 * LEAF // 4 + 5, dtype=torch.float32)       # 4 leaves of bytes, the last one short
    raw = t.numpy().tobytes()
    leaves = b"".join(hashlib.sha256(raw[i:i + LEAF]).digest() for i in range(0, len(raw), LEAF))
    assert leaf_digests(t) == leaves and len(leaves) == 32 * -(-len(raw) // LEAF)
    want = hashlib.sha256(str((str(t.dtype), tuple(t.shape))).encode() + leaves).hexdigest()
    assert sha256tree(t) == want
    t2 = t.clone()
    t2[-1] += 1
    assert sha256tree(t2) != want
