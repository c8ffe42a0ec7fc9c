"""The allocation-free RMSNorm backward, called through its exported C symbol
``sb_rmsnorm_bwd_noalloc`` (for callers that may not allocate device memory on
the call path), must agree with the library's regular RMSNorm backward on two
calls in a row.  This file is collected last on purpose."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry_point():
    import shift_b200._C as C  # loads the library (and PyTorch's runtime it links against)
    lib = ctypes.CDLL(C.__file__)
    fn = lib.sb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return fn


def _close(out, expect, tol=2e-2):
    out, expect = out.float(), expect.float()
    scale = expect.abs().max().item() + 1e-6
    assert (out - expect).abs().max().item() <= tol * scale


def test_noalloc_rmsnorm_bwd_matches_regular_entry_point_twice():
    from shift_b200.ops._ext import ext
    fn = _entry_point()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    for call, (rows, hidden, with_res) in enumerate([(3000, 1024, True), (777, 256, False)]):
        torch.manual_seed(100 + call)
        x = torch.randn(rows, hidden, device=dev).to(torch.bfloat16)
        w = (1 + 0.1 * torch.randn(hidden, device=dev)).to(torch.bfloat16)
        rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
        dy = torch.randn(rows, hidden, device=dev).to(torch.bfloat16)
        dres = torch.randn(rows, hidden, device=dev).to(torch.bfloat16) if with_res else None
        dw_ref = torch.zeros(hidden, device=dev, dtype=torch.float32)
        dx_ref = ext().rmsnorm_bwd(dy, x, rstd, w, dres, dw_ref, False)
        dx = torch.empty_like(x)
        dw = torch.full((hidden,), float("nan"), device=dev, dtype=torch.float32)
        rc = fn(dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), w.data_ptr(),
                dres.data_ptr() if dres is not None else None, dx.data_ptr(), dw.data_ptr(), rows, hidden,
                stream.cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0
        _close(dx, dx_ref)
        _close(dw, dw_ref, tol=1e-3)


def test_noalloc_rejects_unsupported_size_without_launching():
    fn = _entry_point()
    x = torch.zeros(8, 2048, device="cuda", dtype=torch.bfloat16)
    r = torch.zeros(8, device="cuda")
    dw = torch.zeros(2048, device="cuda")
    rc = fn(x.data_ptr(), x.data_ptr(), r.data_ptr(), x.data_ptr(), None, x.data_ptr(), dw.data_ptr(), 8, 2048,
            torch.cuda.current_stream().cuda_stream)
    assert rc == 1


def test_noalloc_rejects_misaligned_or_null_pointers_without_launching():
    fn = _entry_point()
    rows, hidden = 64, 256
    buf = torch.zeros(rows * hidden + 64, device="cuda", dtype=torch.bfloat16)
    x = buf[:rows * hidden]
    off = buf[1:1 + rows * hidden]             # 2 bytes past a 16-byte boundary
    r = torch.ones(rows, device="cuda")
    dw = torch.full((hidden,), 7.0, device="cuda")
    out = torch.full((rows * hidden,), 3.0, device="cuda", dtype=torch.bfloat16)
    s = torch.cuda.current_stream().cuda_stream
    for args in [(off, x, x, out, None), (x, off, x, out, None), (x, x, off, out, None), (x, x, x, off, None),
                 (x, x, x, out, off)]:
        dy, xx, w, dx, dres = args
        rc = fn(dy.data_ptr(), xx.data_ptr(), r.data_ptr(), w.data_ptr(),
                None if dres is None else dres.data_ptr(), dx.data_ptr(), dw.data_ptr(), rows, hidden, s)
        assert rc == 4
    rc = fn(None, x.data_ptr(), r.data_ptr(), x.data_ptr(), None, out.data_ptr(), dw.data_ptr(), rows, hidden, s)
    assert rc == 4
    torch.cuda.synchronize()
    # nothing ran: the outputs still hold their fill values
    assert bool((dw == 7.0).all()) and bool((out == 3.0).all())


def test_noalloc_matches_fp32_statement():
    """dx and dw straight against an fp32 statement of RMSNorm backward."""
    fn = _entry_point()
    dev = torch.device("cuda", 0)
    rows, hidden = 1000, 512
    torch.manual_seed(7)
    x = torch.randn(rows, hidden, device=dev).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(hidden, device=dev)).to(torch.bfloat16)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    dy = torch.randn(rows, hidden, device=dev).to(torch.bfloat16)
    dres = torch.randn(rows, hidden, device=dev).to(torch.bfloat16)
    xf, wf, dyf = x.float(), w.float(), dy.float()
    xhat = xf * rstd[:, None]
    g = dyf * wf
    dx_ref = rstd[:, None] * (g - xhat * (g * xhat).mean(-1, keepdim=True)) + dres.float()
    dw_ref = (dyf * xhat).sum(0)
    dx = torch.empty_like(x)
    dw = torch.empty(hidden, device=dev)
    for _ in range(2):
        rc = fn(dy.data_ptr(), x.data_ptr(), rstd.data_ptr(), w.data_ptr(), dres.data_ptr(), dx.data_ptr(),
                dw.data_ptr(), rows, hidden, torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        assert rc == 0
        _close(dx, dx_ref)
        _close(dw, dw_ref, tol=1e-3)
