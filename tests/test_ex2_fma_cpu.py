"""The FMA-pipe exponential used by the attention forward (``ex2_fma`` in
attention_sm100.cu), restated step for step in float32 numpy: its relative
error against 2^x stays below 1e-4 over the range the softmax feeds it."""
import re
from pathlib import Path

import numpy as np

SRC = Path(__file__).resolve().parents[1] / "shift_b200" / "csrc" / "attention_sm100.cu"


def _coefficients():
    body = SRC.read_text().split("SB_DEVICE float ex2_fma(float x) {", 1)[1].split("}", 1)[0]
    c = [np.float32(v) for v in re.findall(r"(-?\d+\.\d+)f", body.split("const float p =", 1)[1])]
    assert len(c) == 4
    return c            # c3, c2, c1, c0 in the order of the nested fmaf calls


def ex2_fma(x):
    c3, c2, c1, c0 = _coefficients()
    x = np.maximum(x.astype(np.float32), np.float32(-126.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    r = (x - (t - np.float32(12582912.0))).astype(np.float32)
    p = ((c3 * r + c2) * r + c1) * r + c0
    bits = p.astype(np.float32).view(np.int32) + (t.view(np.int32) << np.int32(23))
    return bits.view(np.float32)


def test_relative_error_below_1e_4():
    x = np.linspace(-120.0, 8.0, 2_000_001, dtype=np.float32)
    got = ex2_fma(x).astype(np.float64)
    want = np.exp2(x.astype(np.float64))
    assert np.max(np.abs(got / want - 1.0)) < 1e-4


def test_clamped_tail_is_tiny_and_finite():
    x = np.array([-1e4, -300.0, -126.0, -125.5], dtype=np.float32)
    y = ex2_fma(x)
    assert np.all(np.isfinite(y)) and np.all(y >= 0) and np.all(y < 1e-37)
