"""The allocation-free LayerNorm backward (tnops_ln_bwd_noalloc), called
through its exported C symbol, against the existing entry point
(tnops_ln_bwd with a caller-provided scratch buffer).

The new entry point serves callers that cannot allocate device memory while
they run (fixed-arena engines, C callers without PyTorch's allocator, code
inside another runtime's callbacks); it keeps its scratch in the library.
Two calls in a row, with different sizes, check that what the first call
left in the shared scratch does not leak into the second; both are compared
bit for bit with the existing entry point and against an fp32 PyTorch
autograd LayerNorm backward. Further tests check that calls after the first
leave the device's free memory unchanged and that unsupported widths (C not
a multiple of 4, C above the limit) are refused without a launch.
"""
import ctypes
import os

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

P = ctypes.c_void_p


def _lib():
    lib = ctypes.CDLL(os.path.join(ROOT, "tiny_nccl_b200", "lib", "libtnccl_ops.so"))
    lib.tnops_ln_bwd_noalloc.restype = ctypes.c_int
    lib.tnops_ln_bwd_noalloc.argtypes = [P] * 10 + [ctypes.c_int, ctypes.c_int, P]
    lib.tnops_ln_bwd.restype = ctypes.c_int
    lib.tnops_ln_bwd.argtypes = [P] * 11 + [ctypes.c_int, ctypes.c_int, P]
    lib.tnops_ln_partial_rows.restype = ctypes.c_int
    return lib


def _case(rows, C, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    x = torch.randn(rows, C, device="cuda", generator=g)
    mean = x.mean(-1)
    rstd = torch.rsqrt(x.var(-1, unbiased=False) + 1e-5)
    gy = torch.randn(rows, C, device="cuda", generator=g).to(torch.bfloat16)
    gres = torch.randn(rows, C, device="cuda", generator=g)
    w = 1 + 0.1 * torch.randn(C, device="cuda", generator=g)
    return x, mean, rstd, gy, gres, w


def _outs(rows, C):
    return (torch.empty(rows, C, device="cuda"),
            torch.empty(rows, C, device="cuda", dtype=torch.bfloat16),
            torch.empty(C, device="cuda"), torch.empty(C, device="cuda"))


def _call_noalloc(lib, args, rows, C, stream):
    x, mean, rstd, gy, gres, w = args
    dx, dxb, dw, db = _outs(rows, C)
    rc = lib.tnops_ln_bwd_noalloc(gy.data_ptr(), gres.data_ptr(), x.data_ptr(), w.data_ptr(),
                                  mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dxb.data_ptr(),
                                  dw.data_ptr(), db.data_ptr(), rows, C, stream)
    assert rc == 0
    return dx, dxb, dw, db


def _call_existing(lib, args, rows, C, stream):
    x, mean, rstd, gy, gres, w = args
    dx, dxb, dw, db = _outs(rows, C)
    partial = torch.empty(2 * lib.tnops_ln_partial_rows() * C, device="cuda")
    rc = lib.tnops_ln_bwd(gy.data_ptr(), gres.data_ptr(), x.data_ptr(), w.data_ptr(),
                          mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dxb.data_ptr(),
                          dw.data_ptr(), db.data_ptr(), partial.data_ptr(), rows, C, stream)
    assert rc == 0
    return dx, dxb, dw, db


def _autograd_fp32(args, C):
    """fp32 PyTorch LayerNorm backward of the same forward (eps 1e-5), plus
    the residual-stream gradient."""
    x, _, _, gy, gres, w = args
    xr = x.detach().clone().requires_grad_(True)
    wr = w.detach().clone().requires_grad_(True)
    br = torch.zeros_like(w, requires_grad=True)
    torch.nn.functional.layer_norm(xr, (C,), wr, br, 1e-5).backward(gy.float())
    return xr.grad + gres, wr.grad, br.grad


CASES = [(4096, 768), (333, 1024)]


def test_ln_bwd_noalloc_matches_existing_entry_point(built):
    """Two calls in a row with different sizes: each equals the existing
    entry point (same kernels, so bit for bit) and an fp32 autograd
    LayerNorm backward; what the first call left in the shared scratch does
    not leak into the second."""
    lib = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (rows, C) in enumerate(CASES):
        args = _case(rows, C, seed=call)
        dx, dxb, dw, db = _call_noalloc(lib, args, rows, C, stream)
        rdx, rdxb, rdw, rdb = _call_existing(lib, args, rows, C, stream)
        torch.cuda.synchronize()
        assert torch.equal(dx, rdx) and torch.equal(dxb, rdxb)
        assert torch.equal(dw, rdw) and torch.equal(db, rdb)
        adx, adw, adb = _autograd_fp32(args, C)
        torch.testing.assert_close(dx, adx, rtol=1e-4, atol=1e-4)
        torch.testing.assert_close(dxb.float(), adx, rtol=8e-3, atol=1e-3)  # one bf16 rounding
        torch.testing.assert_close(dw, adw, rtol=1e-4, atol=5e-3)
        torch.testing.assert_close(db, adb, rtol=1e-4, atol=5e-3)


def test_ln_bwd_noalloc_allocates_no_device_memory(built):
    """After one warm-up call per shape (which loads the kernels and looks up
    the scratch address), further calls leave the device's free memory and
    PyTorch's allocator exactly as they were."""
    lib = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    inputs = [(_case(rows, C, seed=7 + i), _outs(rows, C), rows, C)
              for i, (rows, C) in enumerate(CASES)]

    def run_all():
        for (x, mean, rstd, gy, gres, w), (dx, dxb, dw, db), rows, C in inputs:
            rc = lib.tnops_ln_bwd_noalloc(gy.data_ptr(), gres.data_ptr(), x.data_ptr(),
                                          w.data_ptr(), mean.data_ptr(), rstd.data_ptr(),
                                          dx.data_ptr(), dxb.data_ptr(), dw.data_ptr(),
                                          db.data_ptr(), rows, C, stream)
            assert rc == 0

    run_all()
    torch.cuda.synchronize()
    free0, torch0 = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
    for _ in range(3):
        run_all()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0
    assert torch.cuda.memory_allocated() == torch0


def test_ln_bwd_noalloc_rejects_unaligned_width(built):
    lib = _lib()
    rows, C = 16, 770  # C % 4 != 0
    args = _case(rows, C, seed=3)
    x, mean, rstd, gy, gres, w = args
    dx, dxb, dw, db = _outs(rows, C)
    rc = lib.tnops_ln_bwd_noalloc(gy.data_ptr(), gres.data_ptr(), x.data_ptr(), w.data_ptr(),
                                  mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dxb.data_ptr(),
                                  dw.data_ptr(), db.data_ptr(), rows, C,
                                  torch.cuda.current_stream().cuda_stream)
    assert rc != 0


def test_ln_bwd_noalloc_rejects_oversized_rows(built):
    lib = _lib()
    rc = lib.tnops_ln_bwd_noalloc(*([None] * 10), 8, 2048, None)
    assert rc != 0  # cudaErrorInvalidValue, nothing launched
