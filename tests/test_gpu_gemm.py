"""GPU parity of the rotation-accumulate GEMM (FAST and CORDIC modes).

Each output accumulates sequentially over k exactly as the CPU restatement
does (rac_torch/rac_kernels.hip:176-185, 239-425), so the comparison with
oracle.gemm is bit-for-bit.  Against the CORDIC GEMM composed from lib/c's
rac_project_n the bar is normwise max|diff| / rms(ref) <= 1e-4.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

import oracle as O
from rac_b200 import _lib, ext
from rac_b200._lib import LAYOUT_NN, LAYOUT_NT, LAYOUT_TN

pytestmark = pytest.mark.gpu
NORM_TOL = 1e-4


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _normwise(got, ref):
    ref = np.asarray(ref, np.float64)
    return float(np.abs(np.asarray(got, np.float64) - ref).max() / max(math.sqrt(np.mean(ref * ref)), 1e-30))


def _operands(M, N, K, layout, seed):
    rng = np.random.default_rng(seed)
    A = rng.uniform(-1, 1, (K, M) if layout == "tn" else (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (N, K) if layout == "nt" else (K, N)).astype(np.float32)
    return A, B


LAY = {"nn": LAYOUT_NN, "nt": LAYOUT_NT, "tn": LAYOUT_TN}


@pytest.mark.parametrize("layout", ["nn", "nt", "tn"])
@pytest.mark.parametrize("shape", [(1, 1, 1), (63, 65, 67), (127, 255, 131), (128, 128, 128),
                                   (16, 200, 96), (33, 64, 40), (256, 384, 512)])
@pytest.mark.parametrize("mode,iters", [(0, 24), (1, 8), (1, 16), (1, 24), (1, 5)])
def test_gemm_bitexact_vs_restatement(cuda, orc, layout, shape, mode, iters):
    M, N, K = shape
    A, B = _operands(M, N, K, layout, M * 7 + N + K)
    got = ext.gemm(_t(A, cuda), _t(B, cuda), LAY[layout], iters, mode).cpu().numpy()
    want = orc.gemm(A, B, layout, mode, iters)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("iters", [8, 16, 24])
def test_gemm_golden_composed(cuda, golden, iters):
    A, B = golden["mm_A"], golden["mm_B"]
    got = ext.gemm(_t(A, cuda), _t(B, cuda), LAYOUT_NN, iters, 1).cpu().numpy()
    assert _normwise(got, golden[f"mm_cordic{iters}"]) <= NORM_TOL
    got = ext.gemm(_t(A, cuda), _t(B, cuda), LAYOUT_NN, 24, 0).cpu().numpy()
    assert _normwise(got, golden["mm_sgemm"]) <= NORM_TOL


def test_rac_matmul_host_abi_default_knobs(cuda, orc):
    """rac.h rac_matmul with host buffers: process knobs default to CORDIC, 16."""
    L = _lib.lib()
    L.rac_set_cordic_iters(0)
    L.rac_set_cordic_mode(1)
    A, B = _operands(70, 90, 110, "nn", 11)
    C = np.zeros((70, 90), np.float32)
    L.rac_matmul(_p(A), _p(B), _p(C), 70, 90, 110)
    _lib.check()
    assert np.array_equal(C, orc.gemm(A, B, "nn", 1, 16))
    C2 = np.zeros_like(C)
    L.rac_matmul_ex(_p(A), _p(B), _p(C2), 70, 90, 110, 8, 1)
    _lib.check()
    assert np.array_equal(C2, orc.gemm(A, B, "nn", 1, 8))


def test_launchers_alpha_beta(cuda, orc):
    """rac_launch_*_iters: C = alpha*AB + beta*C (rac_kernels.hip:790-797)."""
    L = _lib.lib()
    A, B = _operands(40, 48, 56, "nn", 3)
    C0 = np.random.default_rng(4).standard_normal((40, 48)).astype(np.float32)
    dA, dB, dC = _t(A, cuda), _t(B, cuda), _t(C0, cuda)
    s = torch.cuda.current_stream().cuda_stream
    L.rac_launch_nn_iters(dA.data_ptr(), dB.data_ptr(), dC.data_ptr(), 40, 48, 56,
                          ctypes.c_float(0.5), ctypes.c_float(2.0), 16, 1, s)
    _lib.check()
    acc = orc.gemm(A, B, "nn", 1, 16)
    want = (np.float32(0.5) * acc.astype(np.float64) + 2.0 * C0).astype(np.float32)
    assert np.abs(dC.cpu().numpy() - want).max() <= 1e-6
    dC2 = torch.zeros((40, 48), device=cuda)
    L.rac_launch_nt(dA.data_ptr(), _t(np.ascontiguousarray(B.T), cuda).data_ptr(), dC2.data_ptr(),
                    40, 48, 56, ctypes.c_float(1.0), ctypes.c_float(0.0), s)
    _lib.check()
    assert np.array_equal(dC2.cpu().numpy(), orc.gemm(A, B, "nn", 0, 24))


@pytest.mark.parametrize("act", [1, 2, 3])
def test_fused_bias_act_epilogue(cuda, orc, act):
    A, W = _operands(37, 52, 64, "nt", act)
    bias = np.random.default_rng(9).standard_normal(52).astype(np.float32)
    got = ext.fused_linear_forward(_t(A, cuda), _t(W, cuda), _t(bias, cuda), act, 16, 1).cpu()
    pre = torch.from_numpy(orc.gemm(A, W, "nt", 1, 16)) + torch.from_numpy(bias)
    ref = {1: torch.relu, 2: lambda t: torch.nn.functional.gelu(t), 3: torch.nn.functional.silu}[act](pre)
    assert torch.allclose(got, ref, rtol=1e-5, atol=1e-6)


def test_residual_epilogue_and_strided_operands(cuda, orc):
    A, W = _operands(64, 96, 128, "nt", 21)
    R = np.random.default_rng(1).standard_normal((64, 96)).astype(np.float32)
    got = ext.gemm(_t(A, cuda), _t(W, cuda), LAYOUT_NT, 16, 1, residual=_t(R, cuda)).cpu().numpy()
    want = orc.gemm(A, W, "nt", 1, 16) + R
    assert np.array_equal(got, want.astype(np.float32))
    big = torch.zeros((64, 200), device=cuda)
    big[:, 8:136] = _t(A, cuda)
    view = big[:, 8:136]                                   # leading dim 200, 16B-aligned base
    got2 = ext.gemm(view, _t(W, cuda), LAYOUT_NT, 16, 1).cpu().numpy()
    assert np.array_equal(got2, orc.gemm(A, W, "nt", 1, 16))


def test_large_sampled_rows_vs_oracle(cuda, orc):
    """1024x2048x4096 at 16 iterations: sampled rows bit-exact to the restatement."""
    M, N, K = 1024, 2048, 4096
    g = torch.Generator(device="cpu").manual_seed(5)
    A = (torch.rand((M, K), generator=g) * 2 - 1)
    B = (torch.rand((K, N), generator=g) * 2 - 1)
    C = ext.gemm(A.to(cuda), B.to(cuda), LAYOUT_NN, 16, 1).cpu().numpy()
    An, Bn = A.numpy(), B.numpy()
    for r in (0, 1, 63, 64, 511, 1023):
        assert np.array_equal(C[r:r + 1], orc.gemm(An, Bn, "nn", 1, 16, rows=(r, r + 1))), r


def test_cordic_equals_fast_on_rotated_operand(cuda):
    """Size-independent property: since the direction sequence is data-independent
    and rotation is odd-symmetric, CORDIC(A, B) == FAST(x_n(A)/K(n), B) bit-for-bit.
    Checked at the full 4096^3 benchmark shape."""
    M = N = K = 4096
    g = torch.Generator(device=cuda).manual_seed(0)
    A = torch.rand((M, K), device=cuda, generator=g) * 2 - 1
    B = torch.rand((K, N), device=cuda, generator=g) * 2 - 1
    C = ext.gemm(A, B, LAYOUT_NN, 16, 1)
    # x_n(a)/K(n) for every a: a 1x1 CORDIC GEMM of a against b = 1
    ones = torch.ones((1, 1), device=cuda)
    Ar = ext.gemm(A.reshape(-1, 1), ones, LAYOUT_NN, 16, 1).reshape(M, K)
    Cf = ext.gemm(Ar, B, LAYOUT_NN, 24, 0)
    assert torch.equal(C, Cf)


def test_splitk_skinny_config(cuda, orc):
    """The BASELINE skinny shape M=16, N=11008, K=4096 runs split-K (86 output
    tiles on 148 SMs): normwise <= 1e-4 to the sequential restatement,
    deterministic across calls."""
    M, N, K = 16, 11008, 4096
    rng = np.random.default_rng(16)
    A = rng.uniform(-1, 1, (M, K)).astype(np.float32)
    B = rng.uniform(-1, 1, (K, N)).astype(np.float32)
    dA, dB = _t(A, cuda), _t(B, cuda)
    C1 = ext.gemm(dA, dB, LAYOUT_NN, 16, 1)
    C2 = ext.gemm(dA, dB, LAYOUT_NN, 16, 1)
    assert torch.equal(C1, C2)
    want = orc.gemm(A, B, "nn", 1, 16)
    assert _normwise(C1.cpu().numpy(), want) <= NORM_TOL
    C3 = ext.gemm(dA, dB, LAYOUT_NN, 16, 1, variant=3)      # no split
    assert np.array_equal(C3.cpu().numpy(), want)


@pytest.mark.parametrize("layout", ["nn", "nt", "tn"])
def test_splitk_forced_with_epilogue(cuda, orc, layout):
    M, N, K = 63, 65, 1100
    A, B = _operands(M, N, K, layout, 77)
    bias = np.random.default_rng(3).standard_normal(N).astype(np.float32)
    R = np.random.default_rng(4).standard_normal((M, N)).astype(np.float32)
    kw = dict(bias=_t(bias, cuda), act=3, residual=_t(R, cuda))
    ref = ext.gemm(_t(A, cuda), _t(B, cuda), LAY[layout], 16, 1, variant=1, **kw).cpu().numpy()
    got = ext.gemm(_t(A, cuda), _t(B, cuda), LAY[layout], 16, 1, variant=13, **kw).cpu().numpy()
    assert _normwise(got, ref) <= NORM_TOL
    # and against the CPU oracle: silu(C_orc + R + bias), the epilogue's order
    pre = torch.from_numpy(orc.gemm(A, B, layout, 1, 16)) + torch.from_numpy(R) + torch.from_numpy(bias)
    want = torch.nn.functional.silu(pre).numpy()
    assert _normwise(got, want) <= NORM_TOL
    assert np.array_equal(ref, want) or _normwise(ref, want) <= 1e-6   # unsplit: same k order


@pytest.mark.parametrize("variant", [1, 2, 3, 4])
@pytest.mark.parametrize("layout", ["nn", "nt"])
@pytest.mark.parametrize("iters", [8, 16, 24])
def test_every_tile_variant_bitexact(cuda, orc, variant, layout, iters):
    M, N, K = 200, 328, 256
    A, B = _operands(M, N, K, layout, variant * 31 + iters)
    got = ext.gemm(_t(A, cuda), _t(B, cuda), LAY[layout], iters, 1, variant=variant).cpu().numpy()
    assert np.array_equal(got, orc.gemm(A, B, layout, 1, iters))


@pytest.mark.parametrize("layout", ["nn", "nt", "tn"])
@pytest.mark.parametrize("iters", [4, 8, 16, 24])
@pytest.mark.parametrize("shape", [(63, 65, 67), (128, 96, 160), (16, 200, 96)])
def test_shiftadd_bitexact(cuda, orc, layout, iters, shape):
    """SHIFTADD (rac_kernels.hip:84-122, 217-218): integer shift-add products,
    bit-exact to the CPU restatement."""
    M, N, K = shape
    A, B = _operands(M, N, K, layout, iters + M)
    got = ext.gemm(_t(A, cuda), _t(B, cuda), LAY[layout], iters, 2).cpu().numpy()
    assert np.array_equal(got, orc.gemm(A, B, layout, 2, iters))


def test_shiftadd_edge_values(cuda, orc):
    """Zeros, tiny products flushed to 0, huge products flushed to 0."""
    A = np.array([[0.0, 1e-30, 3e30, -2.5, 1.0]], np.float32)
    B = np.array([[1.0], [1e-20], [4e20], [-0.0], [0.1]], np.float32)
    for it in (1, 8, 24):
        got = ext.gemm(_t(A, cuda), _t(B, cuda), LAYOUT_NN, it, 2).cpu().numpy()
        assert np.array_equal(got, orc.gemm(A, B, "nn", 2, it))


TMA, REGS = 0x100, 0x200      # variant bits: force the TMA / register-staged loader


@pytest.mark.parametrize("variant", [1, 2, 3, 4])
@pytest.mark.parametrize("layout", ["nn", "nt"])
@pytest.mark.parametrize("shape", [(200, 328, 260), (16, 1000, 520), (129, 65, 36)])
def test_tma_staging_bitexact(cuda, orc, variant, layout, shape):
    """cp.async.bulk.tensor staging (4-stage mbarrier pipeline) computes the same
    bits as the register-staged loader and the CPU restatement, including
    out-of-range boxes (M, N not multiples of the tile; K tail)."""
    M, N, K = shape
    A, B = _operands(M, N, K, layout, variant + M)
    dA, dB = _t(A, cuda), _t(B, cuda)
    got = ext.gemm(dA, dB, LAY[layout], 16, 1, variant=TMA | variant).cpu().numpy()
    ref = ext.gemm(dA, dB, LAY[layout], 16, 1, variant=REGS | variant).cpu().numpy()
    assert np.array_equal(got, ref)
    assert np.array_equal(got, orc.gemm(A, B, layout, 1, 16))
    ext.check_device_errors()


def test_tma_staging_splitk_and_strided(cuda, orc):
    M, N, K = 64, 192, 2048
    A, B = _operands(M, N, K, "nn", 5)
    big = torch.zeros((M, K + 16), device=cuda)
    big[:, 4:4 + K] = _t(A, cuda)                      # leading dim K+16, base +16 B
    got = ext.gemm(big[:, 4:4 + K], _t(B, cuda), LAYOUT_NN, 8, 1, variant=TMA | 13).cpu().numpy()
    ref = ext.gemm(_t(A, cuda), _t(B, cuda), LAYOUT_NN, 8, 1, variant=REGS | 13).cpu().numpy()
    assert np.array_equal(got, ref)
    assert _normwise(got, orc.gemm(A, B, "nn", 1, 8)) <= NORM_TOL
    ext.check_device_errors()


@pytest.mark.parametrize("shape", [(1000, 512, 300), (300, 1100, 64), (257, 1030, 40), (2048, 2304, 64)])
def test_rac_matmul_host_pipeline(cuda, orc, shape):
    """rac_matmul with host A and C runs the row-block copy/compute pipeline
    (2 or 4 blocks, ragged); the result equals the restatement bit for bit
    (no split-K at these shapes), with B on the host or on the device."""
    L = _lib.lib()
    M, N, K = shape
    A, B = _operands(M, N, K, "nn", 99)
    want = orc.gemm(A, B, "nn", 1, 16)
    for dev_b in (False, True):
        C = np.zeros((M, N), np.float32)
        Bp = _t(B, cuda) if dev_b else B
        bptr = Bp.data_ptr() if dev_b else _p(B)
        L.rac_matmul_ex(_p(A), bptr, _p(C), M, N, K, 16, 1)
        _lib.check()
        assert np.array_equal(C, want), dev_b


def test_tma_wait_limit_reports_error_and_context_survives(cuda, orc):
    """Failure detection without a fault: with the test hook (variant 0x1000)
    every stage barrier expects 16 bytes more than its copies deliver, so the
    bounded wait runs out; the kernel flags the device error word, the host
    reads RAC_ERR_DEVICE, and the next GEMM on the same context is exact."""
    A, B = _operands(128, 128, 64, "nn", 1)
    dA, dB = _t(A, cuda), _t(B, cuda)
    ext.gemm(dA, dB, LAYOUT_NN, 16, 1, variant=TMA | 0x1000)
    with pytest.raises(_lib.RacError) as e:
        ext.check_device_errors()
    assert e.value.status == -6
    got = ext.gemm(dA, dB, LAYOUT_NN, 16, 1, variant=TMA).cpu().numpy()
    assert np.array_equal(got, orc.gemm(A, B, "nn", 1, 16))
    ext.check_device_errors()


_EDGE = np.array([0.0, -0.0, 1.0, -1.0, 1e-40, -1e-40, 2.0 ** -126, -(2.0 ** -126), 1.5 * 2.0 ** -126,
                  3e38, -3e38, 1e20, -1e20, 1e-20, 0.5, -0.75, 1e-30, 7.0, -123.456], np.float32)


@pytest.mark.skipif(not O.hip_available(), reason="oracle/_ref/librac_hip_mac.so not built")
@pytest.mark.parametrize("mode,iters", [(0, 24), (1, 4), (1, 8), (1, 16), (1, 24), (2, 8), (2, 24)])
def test_gemm_bitexact_vs_reference_hip_code(cuda, mode, iters):
    """Against the reference's own per-MAC code (rac_fma_iters of rac_kernels.hip,
    compiled from the reference file as host code by oracle/build_ref_hip.py):
    random operands in every layout, and every pair of edge values -- zeros,
    subnormals, the smallest normals (where the fused micro-rotation matters),
    huge values -- through a K = 1 GEMM of the edge column against the edge row
    and a K = 2 GEMM that exercises the accumulation."""
    rng = np.random.default_rng(mode * 31 + iters)
    for layout in ("nn", "nt", "tn"):
        A, B = _operands(70, 90, 150, layout, iters)
        got = ext.gemm(_t(A, cuda), _t(B, cuda), LAY[layout], iters, mode).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), O.hip_gemm(A, B, layout, mode, iters).view(np.uint32))
    vals = np.concatenate([_EDGE, rng.standard_normal(13).astype(np.float32)])
    col, row = vals.reshape(-1, 1).copy(), vals.reshape(1, -1).copy()
    got = ext.gemm(_t(col, cuda), _t(row, cuda), LAYOUT_NN, iters, mode).cpu().numpy()
    assert _same_bits(got, O.hip_gemm(col, row, "nn", mode, iters))
    A2 = np.ascontiguousarray(np.stack([vals, vals[::-1]], 1))
    B2 = np.ascontiguousarray(np.stack([vals[::-1], vals], 0))
    got = ext.gemm(_t(A2, cuda), _t(B2, cuda), LAYOUT_NN, iters, mode).cpu().numpy()
    assert _same_bits(got, O.hip_gemm(A2, B2, "nn", mode, iters))


def _same_bits(x, y):
    """Bit-equal, except that any NaN matches any NaN (the GPU's canonical NaN
    and the host's differ in sign and payload) and +0 matches -0: where the
    exact value of a fused multiply-add is a negative number too small to
    represent (e.g. 1e-40 * -1e-40 + 0), IEEE rounding gives -0.0 and the host
    returns -0.0, while the GPU's FFMA returns +0.0 -- equal values, different
    sign bits."""
    zero = (x == 0) & (y == 0)
    return bool(((x.view(np.uint32) == y.view(np.uint32)) | (np.isnan(x) & np.isnan(y)) | zero).all())


@pytest.mark.parametrize("mode,iters", [(0, 24), (1, 16), (1, 8), (2, 8)])
@pytest.mark.parametrize("M,variant", [(96, 0), (16, 0), (70, 13)])
def test_swiglu_epilogue_equals_two_gemms(cuda, mode, iters, M, variant):
    """RAC_ACT_SWIGLU over row-interleaved [gate; up] weights gives the bits of a
    SiLU GEMM on the gate rows times a plain GEMM on the up rows (NT and NN on
    the transposed weights; split-K when M is small or the variant forces it),
    with and without a bias."""
    F_, K = 100, 1300
    rng = np.random.default_rng(M + iters)
    x = _t(rng.uniform(-1, 1, (M, K)).astype(np.float32), cuda)
    wg = _t((rng.standard_normal((F_, K)) * 0.05).astype(np.float32), cuda)
    wu = _t((rng.standard_normal((F_, K)) * 0.05).astype(np.float32), cuda)
    bg = _t(rng.standard_normal(F_).astype(np.float32), cuda)
    bu = _t(rng.standard_normal(F_).astype(np.float32), cuda)
    wgu = torch.stack([wg, wu], 1).reshape(2 * F_, K).contiguous()
    bgu = torch.stack([bg, bu], 1).reshape(2 * F_).contiguous()
    for bias in (False, True):
        g = ext.gemm(x, wg, LAYOUT_NT, iters, mode, act=ext.ACT_SILU, bias=bg if bias else None,
                     variant=variant)
        u = ext.gemm(x, wu, LAYOUT_NT, iters, mode, bias=bu if bias else None, variant=variant)
        want = g * u
        got = ext.gemm(x, wgu, LAYOUT_NT, iters, mode, act=ext.ACT_SWIGLU,
                       bias=bgu if bias else None, variant=variant)
        assert got.shape == (M, F_) and torch.equal(got, want), bias
        got_nn = ext.gemm(x, wgu.t().contiguous(), LAYOUT_NN, iters, mode, act=ext.ACT_SWIGLU,
                          bias=bgu if bias else None, variant=variant)
        assert torch.equal(got_nn, want), bias


@pytest.mark.parametrize("variant", [0, 0x400, 13, 0x2000])
@pytest.mark.parametrize("layout", ["nn", "nt", "tn"])
@pytest.mark.parametrize("shape", [(200, 328, 256), (64, 128, 8), (132, 260, 36)])
def test_fast_kernels_bitexact(cuda, orc, variant, layout, shape):
    """FAST mode: the TMA-staged FFMA2 kernel (NN/TN; 64x128 tiles, or 128x128
    with bit 0x2000), the general one-FFMA kernel (bit 0x400, and NT) and split-K
    (13): the restatement's bits (each FFMA2 half is one fused multiply-add,
    sequential over k)."""
    M, N, K = shape
    A, B = _operands(M, N, K, layout, M + N + K + variant)
    got = ext.gemm(_t(A, cuda), _t(B, cuda), LAY[layout], 24, 0, variant=variant).cpu().numpy()
    want = orc.gemm(A, B, layout, 0, 24)
    if variant == 13:                                 # split-K: a different summation order
        assert _normwise(got, want) <= NORM_TOL
    else:
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
