"""Loader for the in-tree sm_100a extension ``shift_b200._C``.

CUDA tensors always go through the compiled kernels.  If the extension is
missing while a CUDA tensor reaches an op, the op raises: there is no silent
eager fallback on the GPU.  CPU tensors use the fp32 PyTorch restatement of
each op (``shift_b200.ops.reference``), which is also the numerical oracle of
the tests and the compute path of the CPU/gloo harness.
"""
from __future__ import annotations

import importlib
import os
import threading

import torch

_lock = threading.Lock()
_mod = None
_err: Exception | None = None
_status: dict[int, torch.Tensor] = {}


def ext():
    """Return the compiled module or raise with the import error."""
    global _mod, _err
    if _mod is not None:
        return _mod
    with _lock:
        if _mod is None and _err is None:
            try:
                _mod = importlib.import_module("shift_b200._C")
            except Exception as e:  # pragma: no cover - depends on the build
                _err = e
    if _mod is None:
        raise RuntimeError(
            "shift_b200._C (sm_100a kernels) is not built; run `python setup.py build_ext --inplace`"
        ) from _err
    return _mod


def available() -> bool:
    try:
        ext()
        return True
    except RuntimeError:
        return False


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 status words written by bounded waits inside kernels.

    Index 0 is the shared status of the GEMM / attention kernels; 0 means OK,
    1 = an in-CTA pipeline wait ran out, 2 = a peer-flag wait ran out.
    """
    idx = device.index if device.index is not None else torch.cuda.current_device()
    t = _status.get(idx)
    if t is None:
        t = torch.zeros(16, dtype=torch.int32, device=device)
        _status[idx] = t
    return t


def check_status(device: torch.device | None = None) -> int:
    """Read (and clear) the kernel status word; raise on a recorded timeout."""
    dev = device or torch.device("cuda", torch.cuda.current_device())
    s = status_word(dev)
    code = int(s[0].item())
    if code != 0:
        s.zero_()
        raise RuntimeError(f"shift_b200 kernel reported status {code} (bounded wait expired)")
    return code
