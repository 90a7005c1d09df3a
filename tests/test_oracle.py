"""The CPU oracle (oracle/rac_oracle.c) pinned against the reference.

Runs without a GPU: against the committed golden vectors generated from the
reference's own lib/c (tests/golden/make_golden.py), against the reference
library itself when oracle/_ref was built, and against the known-answer
checks of lib/c/test_rac_lib_bvt.c and lib/c/test_rac_lib_dvt.c.
"""
import math

import numpy as np
import pytest


def test_rotate_batch_golden_bitexact(orc, golden):
    out = orc.rotate_batch(golden["rot_v"], golden["rot_theta"], 16, True)
    assert np.array_equal(out.view(np.uint32), golden["rot_batch"].view(np.uint32))


@pytest.mark.parametrize("it", [4, 8, 12, 16, 24])
def test_rotate_project_n_golden_bitexact(orc, golden, it):
    v, th = golden["rot_v"], golden["rot_theta"]
    assert np.array_equal(orc.rotate_batch(v, th, it, False), golden[f"rot_n{it}"])
    assert np.array_equal(orc.project_batch(v, th, it), golden[f"proj_n{it}"])


def test_rope_golden(orc, golden):
    c, s = orc.rope_cache(64, 128, 10000.0)
    assert np.array_equal(c, golden["rope_cos"]) and np.array_equal(s, golden["rope_sin"])
    c2, s2 = orc.rope_cache(4096, 128, 10000.0)
    rows = golden["rope4096_rows"]
    assert np.array_equal(c2[rows], golden["rope4096_cos"])
    assert np.array_equal(s2[rows], golden["rope4096_sin"])
    assert np.array_equal(orc.rope_apply(golden["rope_x"], c, s), golden["rope_out"])


def test_rowwise_golden(orc, golden):
    assert np.array_equal(orc.softmax(golden["softmax_x"]), golden["softmax_out"])
    x, g, b = golden["norm_x"], golden["norm_g"], golden["norm_b"]
    assert np.array_equal(orc.rmsnorm(x, g, 1e-6), golden["rms_out"])
    assert np.array_equal(orc.layernorm(x, g, b, 1e-6), golden["ln_out"])


def test_unary_golden(orc, golden):
    x = golden["unary_x"]
    assert np.array_equal(orc.exp(x), golden["exp_out"])
    assert np.array_equal(orc.tanh(x), golden["tanh_out"])
    L = orc.orc()
    xr = golden["rsqrt_x"]
    assert np.array_equal(np.array([L.orc_rsqrt(float(t)) for t in xr], np.float32), golden["rsqrt_out"])


@pytest.mark.parametrize("it", [8, 16, 24])
def test_cordic_gemm_restatement_vs_composed(orc, golden, it):
    """Sequential rac_fma_cordic GEMM vs the composition from lib/c's rac_project_n."""
    A, B = golden["mm_A"], golden["mm_B"]
    ref = golden[f"mm_cordic{it}"].astype(np.float64)
    got = orc.gemm(A, B, "nn", 1, it)
    rms = math.sqrt(float(np.mean(ref * ref)))
    assert np.abs(got - ref).max() / rms < 1e-5
    # composed in double by the restatement == composed in float by the reference, closely
    assert np.abs(orc.gemm_composed(A, B, it) - ref).max() / rms < 1e-5


def test_fast_gemm_equals_sgemm(orc, golden):
    A, B = golden["mm_A"], golden["mm_B"]
    ref = golden["mm_sgemm"].astype(np.float64)
    got = orc.gemm(A, B, "nn", 0)
    assert np.abs(got - ref).max() / math.sqrt(float(np.mean(ref * ref))) < 1e-5


def test_layouts_agree(orc):
    rng = np.random.default_rng(3)
    A = rng.uniform(-1, 1, (7, 13)).astype(np.float32)
    B = rng.uniform(-1, 1, (13, 5)).astype(np.float32)
    nn = orc.gemm(A, B, "nn", 1, 16)
    assert np.array_equal(nn, orc.gemm(A, np.ascontiguousarray(B.T), "nt", 1, 16))
    assert np.array_equal(nn, orc.gemm(np.ascontiguousarray(A.T), B, "tn", 1, 16))


def test_bvt_known_answers(orc):
    """lib/c/test_rac_lib_bvt.c:164-253 known answers, with that file's tolerances."""
    L = orc.orc()
    ang = np.float32(np.float32(math.pi) * np.float32(0.25))
    v = np.array([[1.0, 0.0]], np.float32)
    expected = math.cos(float(ang))
    r8 = orc.rotate_batch(v, np.array([ang]), 8, False)[0]
    r16 = orc.rotate_batch(v, np.array([ang]), 16, False)[0]
    assert abs(r8[0] - expected) < 0.01 and abs(r16[0] - expected) < 0.001   # :168-173
    s_ = np.zeros(1, np.float32); c_ = np.zeros(1, np.float32)
    import ctypes
    fp = ctypes.POINTER(ctypes.c_float)
    L.orc_sincos(np.float32(math.pi / 2), s_.ctypes.data_as(fp), c_.ctypes.data_as(fp))
    assert abs(s_[0] - 1.0) < 0.01 and abs(c_[0]) < 0.01                     # :175-177
    assert abs(L.orc_rsqrt(4.0) - 0.5) < 1e-6                                # :179-180
    assert L.orc_rsqrt(0.0) == 0.0 and L.orc_rsqrt(-1.0) == 0.0              # :181
    y = orc.layernorm(np.arange(1, 9, dtype=np.float32).reshape(2, 4), None, None, 1e-5)
    assert abs(y[0].mean()) < 0.01 and abs(y[0].var() - 1.0) < 0.05          # :190-204
    y = orc.rmsnorm(np.array([[3.0, 4.0, 0.0, 0.0]], np.float32), None, 1e-6)
    assert abs(y[0, 0] - 1.2) < 0.01 and abs(y[0, 1] - 1.6) < 0.01          # :206-211
    cs, sn = orc.rope_cache(4, 4, 10000.0)
    assert np.all(np.abs(cs[0] - 1.0) < 0.001) and np.all(np.abs(sn[0]) < 0.001)  # :219-221
    x = np.array([1, 2, 3, 4, 5, 6, 7, 8, -1, 0, 0, 1, 0.5, -0.5, 1, -1],
                 np.float32).reshape(1, 1, 4, 4)
    out = orc.rope_apply(x, cs, sn)
    nin = np.hypot(x[..., 0::2], x[..., 1::2])
    nout = np.hypot(out[..., 0::2], out[..., 1::2])
    assert np.all(np.abs(nin - nout) <= 0.01)                                # :232-250


def test_dvt_iteration_bound(orc):
    """lib/c/test_rac_lib_dvt.c:312-337: |rotate_n - libm| <= max(1e-5, 4*2^-n)."""
    rng = np.random.default_rng(42)
    th = rng.uniform(-math.pi, math.pi, 2000).astype(np.float32)
    v = np.tile(np.array([[1.0, 0.0]], np.float32), (th.size, 1))
    for it in range(4, 25, 2):
        r = orc.rotate_batch(v, th, it, False)
        err = max(np.abs(r[:, 0] - np.cos(th)).max(), np.abs(r[:, 1] - np.sin(th)).max())
        assert err <= max(1e-5, 4 * 2.0 ** -it), (it, err)
    p = orc.project_batch(np.array([[1.0, 0.0]], np.float32), np.array([math.pi], np.float32), 8)
    assert abs(p[0] + 1.0) < 0.02                                       # :340-344


def test_gemm_direction_recursion():
    """The d_i sequence hard-wired into the GEMM kernel follows from the atan table."""
    import oracle
    tab = np.ctypeslib.as_array(oracle.orc().orc_atan_table, (24,)) if False else None  # noqa
    atan = np.array([0.78539816, 0.46364761, 0.24497866, 0.12435499, 0.06241881, 0.03123983,
                     0.01562373, 0.00781234, 0.00390623, 0.00195312, 0.00097656, 0.00048828,
                     0.00024414, 0.00012207, 0.00006104, 0.00003052, 0.00001526, 0.00000763,
                     0.00000381, 0.00000191, 0.00000095, 0.00000048, 0.00000024, 0.00000012],
                    np.float32)
    a, ds = np.float32(0.0), []
    for i in range(24):
        d = 1 if a >= 0 else -1
        ds.append(d)
        a = np.float32(a - np.float32(d) * atan[i])
    import ctypes
    from rac_b200 import _lib
    buf = (ctypes.c_int * 24)()
    _lib.lib().rac_b200_cordic_gemm_directions(buf)
    assert list(buf) == ds


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="oracle/_ref not built")
def test_restatement_vs_reference_library_random(orc):
    rng = np.random.default_rng(7)
    v = rng.standard_normal((20000, 2)).astype(np.float32)
    th = rng.uniform(-4, 4, 20000).astype(np.float32)
    assert np.array_equal(orc.rotate_batch(v, th, 16, True), orc.ref_rotate_batch(v, th))
    x = (rng.standard_normal((64, 777)) * 3).astype(np.float32)
    assert np.array_equal(orc.softmax(x), orc.ref_softmax(x))


def test_shiftadd_restatement_properties(orc):
    """rac_shiftadd_mul at 24 bits is the exact product truncated to 24 bits;
    fewer bits never increase |a*b| (rac_kernels.hip:66-83 error model)."""
    L = orc.orc()
    rng = np.random.default_rng(11)
    for a, b in rng.uniform(-4, 4, (500, 2)).astype(np.float32):
        p24 = L.orc_shiftadd_mul(float(a), float(b), 24)
        exact = float(a) * float(b)
        assert abs(p24 - exact) <= abs(exact) * 2 ** -23
        p8 = L.orc_shiftadd_mul(float(a), float(b), 8)
        assert abs(p8) <= abs(p24) and abs(p8 - exact) <= abs(exact) * 2 ** -7


def test_attention_restatement_golden(orc, golden):
    q, k, v, m = golden["att_q"], golden["att_k"], golden["att_v"], golden["att_mask"]
    assert np.array_equal(orc.attention(q, k, v, None, True), golden["att_causal"])
    assert np.array_equal(orc.attention(q, k, v, m, False), golden["att_masked"])


def test_torch_block_restatement_matches_reference_module(block_golden):
    """oracle/torch_block.py against the reference RACLlamaBlock's own output
    (CPU torch, seeded weights, tests/golden/rac_torch_block.npz)."""
    import torch

    from oracle import torch_block as TB
    g = block_golden
    d, H, ff, T, Bt, ms = [int(v) for v in g["cfg"]]
    w = {k[2:]: torch.from_numpy(v) for k, v in g.items() if k.startswith("w.")}
    p = {"norm1": w["norm1.weight"], "qkv": w["attn.qkv.weight"], "out": w["attn.out_proj.weight"],
         "norm2": w["norm2.weight"], "fc1": w["ffn.fc1.weight"], "fc2": w["ffn.fc2.weight"]}
    cos, sin = TB.rope_cache(d // H, ms)
    x = torch.from_numpy(g["x"])
    with torch.no_grad():
        y = TB.block_forward(p, x, H, eps=1e-6, cos=cos, sin=sin, causal=True).numpy()
        y_nc = TB.block_forward(p, x, H, eps=1e-6, cos=cos, sin=sin, causal=False).numpy()
    assert np.abs(y - g["y"]).max() < 1e-5
    assert np.abs(y_nc - g["y_noncausal"]).max() < 1e-5


_HIP = pytest.mark.skipif(not __import__("oracle").hip_available(),
                          reason="oracle/_ref/librac_hip_mac.so not built (no reference checkout)")
# Zeros, subnormals, the normal-range boundary, huge values, infinities, NaN.
_EDGE = np.array([0.0, -0.0, 1.0, -1.0, 1e-40, -1e-40, 2.0 ** -126, -(2.0 ** -126), 3e38, -3e38,
                  1e20, -1e20, 1e-20, 0.5, -0.75, np.inf, -np.inf, np.nan, 1e-30, 7.0, -123.456],
                 np.float32)


def _same_bits(x, y):
    return bool(((x.view(np.int32) == y.view(np.int32)) | (np.isnan(x) & np.isnan(y))).all())


@_HIP
@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("iters", [1, 4, 5, 8, 12, 16, 24])
def test_mac_restatement_equals_reference_hip_code(orc, mode, iters):
    """The restated GEMM (oracle/rac_oracle.c orc_gemm) against a sequential-k GEMM
    over the reference's own rac_fma_iters (rac_kernels.hip:202-218, with
    rac_fma_cordic :176-185 and rac_shiftadd_mul :84-122 compiled from the
    reference file): bit-exact in every layout and on every pair of edge values
    (a K = 1 GEMM of the edge column against the edge row)."""
    rng = np.random.default_rng(100 * mode + iters)
    A = rng.uniform(-1, 1, (33, 47)).astype(np.float32)
    B = (rng.standard_normal((47, 29)) * 3).astype(np.float32)
    for lay in ("nn", "nt", "tn"):
        a = np.ascontiguousarray(A.T) if lay == "tn" else A
        b = np.ascontiguousarray(B.T) if lay == "nt" else B
        assert np.array_equal(orc.gemm(a, b, lay, mode, iters), orc.hip_gemm(a, b, lay, mode, iters))
    # Edge values.  The restatement rounds the micro-rotation's product c*y on its
    # own, the HIP build fuses it: they differ only where c*y is subnormal, i.e. for
    # |a| within 2^24 of the smallest normal at iters >= 16 -- a regime the GPU
    # kernels match the reference's fused form in (tests/test_gpu_gemm.py).
    vals = np.concatenate([_EDGE, rng.standard_normal(24).astype(np.float32)])
    col, row = vals.reshape(-1, 1).copy(), vals.reshape(1, -1).copy()
    want = orc.hip_gemm(col, row, "nn", mode, iters)
    got = orc.gemm(col, row, "nn", mode, iters)
    normal_a = (np.abs(vals) >= 2.0 ** -102) | (vals == 0) | ~np.isfinite(vals)
    assert _same_bits(got[normal_a], want[normal_a])
    if mode != 1:
        assert _same_bits(got, want)


@_HIP
@pytest.mark.parametrize("iters", [1, 4, 8, 16, 24])
def test_shiftadd_restatement_equals_reference_hip_code(orc, iters):
    """orc_shiftadd_mul bit for bit against the reference's rac_shiftadd_mul on
    50k random pairs spanning 2^-100 .. 2^100 (flush-to-zero and overflow
    included), and its MAC (acc + product) through rac_fma_iters."""
    rng = np.random.default_rng(iters)
    n = 50000
    a = (rng.standard_normal(n) * 2.0 ** rng.integers(-100, 100, n)).astype(np.float32)
    b = (rng.standard_normal(n) * 2.0 ** rng.integers(-100, 100, n)).astype(np.float32)
    acc = rng.standard_normal(n).astype(np.float32)
    L = orc.orc()
    mine = np.array([L.orc_shiftadd_mul(float(x), float(y), iters) for x, y in zip(a[:5000], b[:5000])],
                    np.float32)
    theirs = np.array([orc.hip().hipref_shiftadd_mul(float(x), float(y), iters)
                       for x, y in zip(a[:5000], b[:5000])], np.float32)
    assert _same_bits(mine, theirs)
    prod = np.array([L.orc_shiftadd_mul(float(x), float(y), iters) for x, y in zip(a, b)], np.float32)
    assert _same_bits(orc.hip_mac(a, b, acc, iters, 2), (acc + prod).astype(np.float32))


def test_cordic_operand_identity(orc):
    """CORDIC(A, B) == FAST(r(A), B) bit for bit, r = oracle.cordic_operand: the
    identity the block-level CORDIC oracle rests on."""
    rng = np.random.default_rng(5)
    A = rng.uniform(-1, 1, (40, 300)).astype(np.float32)
    B = rng.uniform(-1, 1, (300, 24)).astype(np.float32)
    for it in (8, 16, 24):
        assert np.array_equal(orc.gemm(A, B, "nn", 1, it), orc.gemm(orc.cordic_operand(A, it), B, "nn", 0, it))
