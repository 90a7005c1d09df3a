"""rac_gemm_splitk_noalloc_async: the GEMM entry point that allocates nothing.

It is meant for callers that cannot let the library allocate device memory
(a host with a fixed, fully accounted memory budget per plugin, or a
latency-critical path where an allocation could stall), so it keeps the
split-K partial sums in a fixed array inside the library.  These tests call
it through the C ABI and compare it with rac_gemm_async, the entry point
that takes its workspace from the stream-ordered pool, on two calls in a row
(the second with new inputs, so stale scratch contents would show), and
check that a problem larger than the array is refused with an error.

The file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from rac_b200 import _lib

pytestmark = pytest.mark.gpu
NORM_TOL = 1e-4          # the GEMM bar used throughout tests/


def _normwise(got, ref):
    got = got.double()
    ref = ref.double()
    return float((got - ref).abs().max() / max(math.sqrt(float((ref * ref).mean())), 1e-30))


def _call(name, A, B, C, M, N, K, layout, mode, iters, extra, stream):
    L = _lib.lib()
    lda = A.stride(0)
    ldb = B.stride(0)
    args = [A.data_ptr(), lda, B.data_ptr(), ldb, C.data_ptr(), C.stride(0), None, 0, None,
            M, N, K, layout, mode, iters, ctypes.c_float(1.0), ctypes.c_float(0.0), 0]
    return getattr(L, name)(*args, *extra, stream)


@pytest.mark.parametrize("layout,mode,iters", [(0, 1, 16), (1, 1, 8), (0, 0, 24), (2, 1, 5)])
def test_noalloc_matches_pooled_entry_point_twice(cuda, layout, mode, iters):
    M, N, K = 16, 11008, 4096
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=cuda).manual_seed(layout * 10 + iters)
    for call in range(2):
        A = torch.rand((K, M) if layout == 2 else (M, K), device=cuda, generator=g) * 2 - 1
        B = torch.rand((N, K) if layout == 1 else (K, N), device=cuda, generator=g) * 2 - 1
        C_ref = torch.empty((M, N), device=cuda)
        C_new = torch.full((M, N), float("nan"), device=cuda)
        st = _call("rac_gemm_async", A, B, C_ref, M, N, K, layout, mode, iters, [0], s)
        _lib.check(st)
        st = _call("rac_gemm_splitk_noalloc_async", A, B, C_new, M, N, K, layout, mode, iters, [0], s)
        _lib.check(st)
        torch.cuda.synchronize()
        assert _normwise(C_new, C_ref) <= NORM_TOL, call


def test_noalloc_rejects_problems_larger_than_its_array(cuda):
    M, N, K = 2048, 2048, 1024                 # 2 splits x 4 Mi floats > 4 Mi
    A = torch.zeros((M, K), device=cuda)
    B = torch.zeros((K, N), device=cuda)
    C = torch.zeros((M, N), device=cuda)
    st = _call("rac_gemm_splitk_noalloc_async", A, B, C, M, N, K, 0, 1, 16, [2],
               torch.cuda.current_stream().cuda_stream)
    assert st == -2
    assert "scratch" in _lib.lib().rac_last_error_string().decode()
