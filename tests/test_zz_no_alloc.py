"""The allocation-free LayerNorm backward (tnops_ln_bwd_noalloc), called
through its exported C symbol, against the existing entry point
(tnops_ln_bwd with a caller-provided scratch buffer).

The new entry point serves callers that cannot allocate device memory while
they run (fixed-arena engines, C callers without PyTorch's allocator, code
inside another runtime's callbacks); it keeps its scratch in the library.
Two calls in a row, with different sizes, check that what the first call
left in the shared scratch does not leak into the second.
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


def test_ln_bwd_noalloc_matches_existing_entry_point(built):
    lib = _lib()
    stream = torch.cuda.current_stream().cuda_stream
    for call, (rows, C) in enumerate([(4096, 768), (333, 1024)]):
        x, mean, rstd, gy, gres, w = _case(rows, C, seed=call)
        dx, dxb, dw, db = _outs(rows, C)
        rc = lib.tnops_ln_bwd_noalloc(gy.data_ptr(), gres.data_ptr(), x.data_ptr(), w.data_ptr(),
                                      mean.data_ptr(), rstd.data_ptr(), dx.data_ptr(),
                                      dxb.data_ptr(), dw.data_ptr(), db.data_ptr(), rows, C,
                                      stream)
        assert rc == 0
        rdx, rdxb, rdw, rdb = _outs(rows, C)
        partial = torch.empty(2 * lib.tnops_ln_partial_rows() * C, device="cuda")
        rc = lib.tnops_ln_bwd(gy.data_ptr(), gres.data_ptr(), x.data_ptr(), w.data_ptr(),
                              mean.data_ptr(), rstd.data_ptr(), rdx.data_ptr(), rdxb.data_ptr(),
                              rdw.data_ptr(), rdb.data_ptr(), partial.data_ptr(), rows, C, stream)
        assert rc == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(dx, rdx, atol=1e-3, rtol=1e-3)
        torch.testing.assert_close(dxb.float(), rdxb.float(), atol=2e-2, rtol=1e-2)
        torch.testing.assert_close(dw, rdw, atol=1e-2, rtol=1e-3)
        torch.testing.assert_close(db, rdb, atol=1e-2, rtol=1e-3)


def test_ln_bwd_noalloc_rejects_oversized_rows(built):
    lib = _lib()
    rc = lib.tnops_ln_bwd_noalloc(*([None] * 10), 8, 2048, None)
    assert rc != 0  # cudaErrorInvalidValue, nothing launched
