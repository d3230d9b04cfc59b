"""The allocation-free RMSNorm backward entry point, called through its exported C symbol.

Callers that cannot allocate device memory (their host framework owns every allocation, or they must not let
a call grow the memory footprint) use ``emb_rmsnorm_bwd_noalloc``; it keeps its partial sums in a fixed
device array built into the library.  This test checks it against the regular ``rmsnorm_bwd`` entry point on
two calls in a row (the second call reuses the scratch the first one left behind).  It sits in its own file,
collected last, so a run that stops at the first failure has already run every other test.
"""
import ctypes
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _symbol():
    from elasticmegatron_b200 import _C  # loads the library and its torch dependencies

    lib = ctypes.CDLL(_C.__file__)
    fn = lib.emb_rmsnorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    return fn


def _call(fn, dy, x, w, rstd, dx, dw, accumulate):
    T, H = x.shape
    stream = torch.cuda.current_stream().cuda_stream
    return fn(dy.data_ptr(), x.data_ptr(), w.data_ptr(), rstd.data_ptr(), dx.data_ptr(), dw.data_ptr(), T, H,
              accumulate, stream)


@pytest.mark.parametrize("T,H", [(1024, 4096), (257, 512)])
def test_noalloc_matches_regular_entry_point(T, H):
    from elasticmegatron_b200.ops.native import ext

    fn = _symbol()
    torch.manual_seed(0)
    for call in range(2):
        x = torch.randn(T, H, device="cuda").bfloat16()
        w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
        dy = torch.randn(T, H, device="cuda").bfloat16()
        _, rstd = ext().rmsnorm_fwd(x, w, 1e-5)
        dx_ref, dw_ref = ext().rmsnorm_bwd(dy, x, w, rstd)
        dx = torch.empty_like(x)
        dw = torch.full((H,), float("nan"), device="cuda")
        assert _call(fn, dy, x, w, rstd, dx, dw, 0) == 0
        torch.cuda.synchronize()
        tol = 5e-2 * math.sqrt(T / 64)
        torch.testing.assert_close(dx.float(), dx_ref.float(), atol=3e-2, rtol=3e-2)
        torch.testing.assert_close(dw, dw_ref, atol=tol, rtol=1e-2)
        # accumulate mode adds into the caller's buffer
        acc = torch.ones(H, device="cuda")
        assert _call(fn, dy, x, w, rstd, dx, acc, 1) == 0
        torch.cuda.synchronize()
        torch.testing.assert_close(acc, dw_ref + 1, atol=tol, rtol=1e-2)


def test_noalloc_rejects_oversized_shapes():
    fn = _symbol()
    x = torch.zeros(8, 8, device="cuda").bfloat16()
    r = fn(x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), x.data_ptr(), 8, 40000, 0,
           torch.cuda.current_stream().cuda_stream)
    assert r == -22
