"""rac_gemm_splitk_noalloc_async: the GEMM entry point that allocates nothing.

It is meant for callers that cannot let the library allocate device memory
(a host with a fixed, fully accounted memory budget per plugin, or a
latency-critical path where an allocation could stall), so it keeps the
split-K partial sums in a fixed array inside the library.  These tests call
it through the C ABI and compare it with rac_gemm_async, the entry point
that takes its workspace from the stream-ordered pool, on two calls in a row
(the second with new inputs, so stale scratch contents would show) and
require the same bits -- both run the same kernels and the same split-K
reduction -- with and without an epilogue (beta, input C, bias, SiLU); sampled
rows are also held to the CPU oracle.  A problem larger than the array must
be refused with an error.

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
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(got - ref).max() / max(math.sqrt(float((ref * ref).mean())), 1e-30))


def _call(name, A, B, C, M, N, K, layout, mode, iters, last, stream, Cin=None, bias=None,
          beta=0.0, act=0):
    L = _lib.lib()
    args = [A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0), C.data_ptr(), C.stride(0),
            None if Cin is None else Cin.data_ptr(), 0 if Cin is None else Cin.stride(0),
            None if bias is None else bias.data_ptr(),
            M, N, K, layout, mode, iters, ctypes.c_float(1.0), ctypes.c_float(beta), act]
    return getattr(L, name)(*args, last, stream)


@pytest.mark.parametrize("layout,mode,iters", [(0, 1, 16), (1, 1, 8), (0, 0, 24), (2, 1, 5)])
def test_noalloc_matches_pooled_entry_point_twice(cuda, orc, layout, mode, iters):
    """Automatic split count: both entry points pick the same S and run the same
    kernels, so the outputs must be equal bit for bit; two calls in a row with
    fresh inputs (and an output pre-filled with NaN) so that stale scratch or an
    unwritten element would show.  Sampled rows also against the CPU oracle."""
    M, N, K = 16, 11008, 4096
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=cuda).manual_seed(layout * 10 + iters)
    for call in range(2):
        A = torch.rand((K, M) if layout == 2 else (M, K), device=cuda, generator=g) * 2 - 1
        B = torch.rand((N, K) if layout == 1 else (K, N), device=cuda, generator=g) * 2 - 1
        C_ref = torch.empty((M, N), device=cuda)
        C_new = torch.full((M, N), float("nan"), device=cuda)
        _lib.check(_call("rac_gemm_async", A, B, C_ref, M, N, K, layout, mode, iters, 0, s))
        _lib.check(_call("rac_gemm_splitk_noalloc_async", A, B, C_new, M, N, K, layout, mode,
                         iters, 0, s))
        torch.cuda.synchronize()
        assert torch.equal(C_new, C_ref), call
        want = orc.gemm(A.cpu().numpy(), B.cpu().numpy(), ("nn", "nt", "tn")[layout], mode, iters,
                        rows=(3, 5))
        assert _normwise(C_new[3:5].cpu().numpy(), want) <= NORM_TOL, call


@pytest.mark.parametrize("layout", [0, 1, 2])
def test_noalloc_explicit_splits_with_epilogue(cuda, layout):
    """splits = 3 with beta != 0, an input C, a bias and SiLU: the same bits as the
    pooled entry point forced to 3 splits (variant 13), which applies the same
    epilogue in the same split-K reduction kernel; twice, with new inputs."""
    M, N, K = 70, 300, 1500
    s = torch.cuda.current_stream().cuda_stream
    g = torch.Generator(device=cuda).manual_seed(40 + layout)
    for call in range(2):
        A = torch.rand((K, M) if layout == 2 else (M, K), device=cuda, generator=g) * 2 - 1
        B = torch.rand((N, K) if layout == 1 else (K, N), device=cuda, generator=g) * 2 - 1
        Cin = torch.randn((M, N), device=cuda, generator=g)
        bias = torch.randn((N,), device=cuda, generator=g)
        C_ref = torch.empty((M, N), device=cuda)
        C_new = torch.full((M, N), float("nan"), device=cuda)
        kw = dict(Cin=Cin, bias=bias, beta=0.5, act=3)
        _lib.check(_call("rac_gemm_async", A, B, C_ref, M, N, K, layout, 1, 16, 13, s, **kw))
        _lib.check(_call("rac_gemm_splitk_noalloc_async", A, B, C_new, M, N, K, layout, 1, 16, 3, s,
                         **kw))
        torch.cuda.synchronize()
        assert torch.equal(C_new, C_ref), call
        assert torch.isfinite(C_new).all()


def test_noalloc_rejects_problems_larger_than_its_array(cuda):
    M, N, K = 2048, 2048, 1024                 # 2 splits x 4 Mi floats > 4 Mi
    A = torch.zeros((M, K), device=cuda)
    B = torch.zeros((K, N), device=cuda)
    C = torch.zeros((M, N), device=cuda)
    st = _call("rac_gemm_splitk_noalloc_async", A, B, C, M, N, K, 0, 1, 16, 2,
               torch.cuda.current_stream().cuda_stream)
    assert st == -2
    assert "scratch" in _lib.lib().rac_last_error_string().decode()
