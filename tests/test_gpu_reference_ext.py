"""The FAST-mode GEMM against the reference's own CUDA kernels.

oracle/build_ref_cuda.py compiles the reference PyTorch extension
(rac_torch/rac_torch.cu, module rac_cuda_ext) from its sources for sm_100a
into oracle/_ref/.  Its GEMMs multiply with the sign-XOR FMA (rac_fma,
rac_torch.cu) and accumulate over k in order per output, as this library's
FAST mode does, so the results must be equal bit for bit: matmul_forward
(NN, tiers small / micro4 / micro8 by size) and linear_forward (x W^T, NT).
The same-GPU timing at 4096^3 is the "reference kernel rebuilt for this GPU"
comparison; this library must be faster.
"""
import importlib.util
import os

import pytest
import torch

from rac_b200 import ext
from rac_b200._lib import LAYOUT_NN, LAYOUT_NT

pytestmark = pytest.mark.gpu
SO = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                  "rac_cuda_ext.so")


@pytest.fixture(scope="module")
def ref_ext(cuda):
    if not os.path.exists(SO):
        pytest.skip("oracle/_ref/rac_cuda_ext.so not built (python -m oracle.build_ref_cuda)")
    spec = importlib.util.spec_from_file_location("rac_cuda_ext", SO)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("shape", [(64, 64, 64), (300, 260, 128), (1000, 1000, 1000), (4096, 4096, 4096)])
def test_fast_gemm_equals_reference_cuda_kernels(cuda, ref_ext, shape):
    M, N, K = shape
    g = torch.Generator(device=cuda).manual_seed(M + N + K)
    A = torch.rand((M, K), device=cuda, generator=g) * 2 - 1
    B = torch.rand((K, N), device=cuda, generator=g) * 2 - 1
    assert torch.equal(ref_ext.matmul_forward(A, B), ext.gemm(A, B, LAYOUT_NN, 24, 0))
    W = B.t().contiguous()
    assert torch.equal(ref_ext.linear_forward(A, W, torch.empty(0, device=cuda)),
                       ext.gemm(A, W, LAYOUT_NT, 24, 0))


def _ms(fn, reps=10):
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def test_faster_than_reference_cuda_kernels(cuda, ref_ext):
    M = N = K = 4096
    A = torch.rand((M, K), device=cuda) * 2 - 1
    B = torch.rand((K, N), device=cuda) * 2 - 1
    W = B.t().contiguous()
    empty = torch.empty(0, device=cuda)
    t = {"ref_nn": _ms(lambda: ref_ext.matmul_forward(A, B)),
         "ours_nn": _ms(lambda: ext.gemm(A, B, LAYOUT_NN, 24, 0)),
         "ref_nt": _ms(lambda: ref_ext.linear_forward(A, W, empty)),
         "ours_nt": _ms(lambda: ext.gemm(A, W, LAYOUT_NT, 24, 0))}
    print({k: f"{v:.3f} ms, {2 * M * N * K / v / 1e9:.1f} TFLOP/s" for k, v in t.items()})
    assert t["ours_nn"] < t["ref_nn"] and t["ours_nt"] < t["ref_nt"]
