"""CPU oracle for the RAC hot path -- TEST INFRASTRUCTURE ONLY.

Two checkers live here:

* ``orc``: the C restatement in ``rac_oracle.c`` (liborc.so), each function
  citing the reference routine it follows.
* ``ref``: the reference's own ``lib/c`` compiled from its sources by
  ``oracle/Makefile`` into ``oracle/_ref/librac_ref.so`` (absent when it was
  never built; the GPU box receives the prebuilt file).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU legs of ``bench.py``
import this package; the ``rac_b200`` product never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORC_PATH = os.path.join(HERE, "liborc.so")
REF_PATH = os.path.join(HERE, "_ref", "librac_ref.so")

_fp = C.POINTER(C.c_float)


class Vec2(C.Structure):
    _fields_ = [("x", C.c_float), ("y", C.c_float)]


REF_PY_DIR = os.path.join(HERE, "_ref", "py")
HIP_PATH = os.path.join(HERE, "_ref", "librac_hip_mac.so")


def build() -> None:
    """Compile liborc.so; where the reference checkout exists, also the reference's
    lib/c (Makefile), its per-MAC HIP arithmetic as host code (build_ref_hip), a
    copy of its Python module rac_torch.py under _ref/py/ (run on this library by
    the drop-in test, and on the CPU as the block's timed baseline), and its CUDA
    extension (only when not built yet, ~3 minutes)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    from . import build_ref_hip
    build_ref_hip.build()
    src = os.path.join(build_ref_hip.default_root(), "rac_torch", "rac_torch.py")
    if os.path.exists(src):
        import shutil
        os.makedirs(REF_PY_DIR, exist_ok=True)
        shutil.copyfile(src, os.path.join(REF_PY_DIR, "rac_torch_ref.py"))
    if not os.path.exists(os.path.join(HERE, "_ref", "rac_cuda_ext.so")):
        from . import build_ref_cuda
        try:
            build_ref_cuda.build()
        except Exception as e:          # the parity test skips without it
            print(f"oracle: reference CUDA extension not built: {e}")


def _p(a: np.ndarray):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return a.ctypes.data_as(_fp)


_orc = None
_ref = None


def orc() -> C.CDLL:
    global _orc
    if _orc is None:
        if not os.path.exists(ORC_PATH):
            build()
        lib = C.CDLL(ORC_PATH)
        L, I, F = C.c_long, C.c_int, C.c_float
        lib.orc_rotate_batch.argtypes = [_fp, _fp, _fp, L, I, I]
        lib.orc_project_batch.argtypes = [_fp, _fp, _fp, L, I]
        lib.orc_project_n.argtypes = [F, F, F, I]
        lib.orc_project_n.restype = F
        lib.orc_sincos.argtypes = [F, _fp, _fp]
        lib.orc_rope_cache.argtypes = [_fp, _fp, I, I, F]
        lib.orc_rope_apply.argtypes = [_fp, _fp, _fp, I, I, I, I]
        lib.orc_softmax_batch.argtypes = [_fp, _fp, L, I]
        lib.orc_rmsnorm.argtypes = [_fp, _fp, _fp, F, L, I]
        lib.orc_layernorm.argtypes = [_fp, _fp, _fp, _fp, F, L, I]
        lib.orc_exp_batch.argtypes = [_fp, _fp, L]
        lib.orc_tanh_batch.argtypes = [_fp, _fp, L]
        lib.orc_rsqrt.argtypes = [F]
        lib.orc_rsqrt.restype = F
        lib.orc_gemm.argtypes = [_fp, _fp, _fp, I, I, I, I, I, I, L, L]
        lib.orc_attention.argtypes = [_fp, _fp, _fp, _fp, I, _fp, I, I, I, I]
        lib.orc_shiftadd_mul.argtypes = [F, F, I]
        lib.orc_shiftadd_mul.restype = F
        lib.orc_gemm_composed.argtypes = [_fp, _fp, _fp, I, I, I, I, L, L]
        lib.orc_gemm_composed_with.argtypes = [C.c_void_p, _fp, _fp, _fp, I, I, I, I, L, L]
        lib.orc_num_threads.restype = I
        _orc = lib
    return _orc


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


def ref() -> C.CDLL:
    """The reference lib/c (loaded RTLD_LOCAL: its rac_* names stay private)."""
    global _ref
    if _ref is None:
        lib = C.CDLL(REF_PATH, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        I, F = C.c_int, C.c_float
        lib.rac_rotate.argtypes = [Vec2, F]
        lib.rac_rotate.restype = Vec2
        lib.rac_rotate_n.argtypes = [Vec2, F, I]
        lib.rac_rotate_n.restype = Vec2
        lib.rac_project_n.argtypes = [Vec2, F, I]
        lib.rac_project_n.restype = F
        lib.rac_rotate_batch.argtypes = [_fp, _fp, _fp, I]
        lib.rac_sincos.argtypes = [F, _fp, _fp]
        lib.rac_rsqrt.argtypes = [F]
        lib.rac_rsqrt.restype = F
        lib.rac_exp.argtypes = [F]
        lib.rac_exp.restype = F
        lib.rac_tanh.argtypes = [F]
        lib.rac_tanh.restype = F
        lib.rac_softmax_batch.argtypes = [_fp, _fp, I, I]
        lib.rac_rmsnorm.argtypes = [_fp, _fp, _fp, F, I, I, C.c_void_p]
        lib.rac_rmsnorm.restype = I
        lib.rac_layernorm.argtypes = [_fp, _fp, _fp, _fp, F, I, I, C.c_void_p]
        lib.rac_layernorm.restype = I
        lib.rac_rope_cache.argtypes = [_fp, _fp, I, I, F]
        lib.rac_rope_cache.restype = I
        lib.rac_rope_apply.argtypes = [_fp, _fp, _fp, I, I, I, I, C.c_void_p]
        lib.rac_rope_apply.restype = I
        lib.rac_hal_sgemm.argtypes = [_fp, _fp, _fp, I, I, I, F, F]
        lib.rac_hal_sgemm.restype = I
        lib.rac_sgemm.argtypes = [_fp, _fp, _fp, I, I, I, F, F, C.c_void_p]
        lib.rac_sgemm.restype = I
        lib.rac_alu_rotate_batch.argtypes = [_fp, _fp, _fp, I]
        _ref = lib
    return _ref


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ── numpy front-ends of the restatement ────────────────────────────────────

def rotate_batch(v, theta, iters: int = 16, literal_kinv: bool = True):
    """v: [n, 2] float32; returns [n, 2]. literal_kinv -> rac_rotate_batch."""
    v, theta = _f32(v), _f32(theta)
    out = np.empty_like(v)
    orc().orc_rotate_batch(_p(v), _p(theta), _p(out), theta.size, iters, int(literal_kinv))
    return out


def project_batch(v, theta, iters: int = 16):
    v, theta = _f32(v), _f32(theta)
    out = np.empty_like(theta)
    orc().orc_project_batch(_p(v), _p(theta), _p(out), theta.size, iters)
    return out


def rope_cache(max_seq: int, head_dim: int, base: float = 10000.0):
    c = np.empty((max_seq, head_dim // 2), np.float32)
    s = np.empty_like(c)
    orc().orc_rope_cache(_p(c), _p(s), max_seq, head_dim, base)
    return c, s


def rope_apply(x, cos_tab, sin_tab):
    x = _f32(x).copy()
    b, h, s, hd = x.shape
    orc().orc_rope_apply(_p(x), _p(_f32(cos_tab)), _p(_f32(sin_tab)), b, h, s, hd)
    return x


def softmax(x):
    x = _f32(x)
    out = np.empty_like(x)
    orc().orc_softmax_batch(_p(x), _p(out), x.size // x.shape[-1], x.shape[-1])
    return out


def rmsnorm(x, gamma=None, eps: float = 1e-6):
    x = _f32(x)
    y = np.empty_like(x)
    g = _p(_f32(gamma)) if gamma is not None else None
    orc().orc_rmsnorm(_p(x), _p(y), g, eps, x.size // x.shape[-1], x.shape[-1])
    return y


def layernorm(x, gamma=None, beta=None, eps: float = 1e-6):
    x = _f32(x)
    y = np.empty_like(x)
    g = _p(_f32(gamma)) if gamma is not None else None
    b = _p(_f32(beta)) if beta is not None else None
    orc().orc_layernorm(_p(x), _p(y), g, b, eps, x.size // x.shape[-1], x.shape[-1])
    return y


def exp(x):
    x = _f32(x)
    y = np.empty_like(x)
    orc().orc_exp_batch(_p(x), _p(y), x.size)
    return y


def tanh(x):
    x = _f32(x)
    y = np.empty_like(x)
    orc().orc_tanh_batch(_p(x), _p(y), x.size)
    return y


LAYOUTS = {"nn": 0, "nt": 1, "tn": 2}


def gemm(A, B, layout: str = "nn", mode: int = 1, iters: int = 16, rows=None):
    """Sequential-k GEMM of rac_kernels.hip (mode 0 FAST, 1 CORDIC, 2 SHIFTADD).

    Shapes: nn A[M,K] B[K,N]; nt A[M,K] B[N,K]; tn A[K,M] B[K,N].
    rows=(r0, r1) computes only output rows [r0, r1)."""
    A, B = _f32(A), _f32(B)
    lay = LAYOUTS[layout]
    if lay == 2:
        K, M = A.shape
    else:
        M, K = A.shape
    N = B.shape[0] if lay == 1 else B.shape[1]
    r0, r1 = rows if rows is not None else (0, M)
    C_ = np.empty((r1 - r0, N), np.float32)
    orc().orc_gemm(_p(A), _p(B), _p(C_), M, N, K, lay, mode, iters, r0, r1)
    return C_


def attention(q, k, v, mask=None, is_causal=False):
    """rac_scaled_dot_attention restated; q, k, v: [b, h, s, hd]."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty_like(q)
    m = _p(_f32(mask)) if mask is not None else None
    b, h, s, hd = q.shape
    orc().orc_attention(_p(q), _p(k), _p(v), m, int(is_causal), _p(out), b, h, s, hd)
    return out


def ref_attention(q, k, v, mask=None, is_causal=False):
    """The reference library's own rac_scaled_dot_attention."""
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty_like(q)
    L = ref()
    L.rac_scaled_dot_attention.argtypes = [_fp, _fp, _fp, _fp, C.c_int, _fp, C.c_int, C.c_int,
                                           C.c_int, C.c_int, C.c_void_p]
    L.rac_scaled_dot_attention.restype = C.c_int
    b, h, s, hd = q.shape
    m = _p(_f32(mask)) if mask is not None else None
    assert L.rac_scaled_dot_attention(_p(q), _p(k), _p(v), m, int(is_causal), _p(out), b, h, s, hd, None) == 0
    return out


def gemm_composed(A, B, iters: int = 16, rows=None):
    """CORDIC GEMM composed from rac_project_n, double accumulation (NN)."""
    A, B = _f32(A), _f32(B)
    M, K = A.shape
    N = B.shape[1]
    r0, r1 = rows if rows is not None else (0, M)
    C_ = np.empty((r1 - r0, N), np.float32)
    orc().orc_gemm_composed(_p(A), _p(B), _p(C_), M, N, K, iters, r0, r1)
    return C_


def gemm_composed_ref(A, B, iters: int = 16, rows=None):
    """CORDIC GEMM composed from the REFERENCE library's rac_project_n."""
    A, B = _f32(A), _f32(B)
    M, K = A.shape
    N = B.shape[1]
    r0, r1 = rows if rows is not None else (0, M)
    C_ = np.empty((r1 - r0, N), np.float32)
    fn = C.cast(ref().rac_project_n, C.c_void_p)
    orc().orc_gemm_composed_with(fn, _p(A), _p(B), _p(C_), M, N, K, iters, r0, r1)
    return C_


def cordic_operand(a, iters: int = 16):
    """r(a) = round(x_n(a) * (1/K(n))) elementwise: the CORDIC-mode MAC is
    fmaf(r(a), b, acc) exactly (the directions do not depend on the data and
    the rotation is odd), so a CORDIC GEMM is a FAST GEMM of r(A) and B.
    Computed as a 1x1 restated CORDIC GEMM against b = 1."""
    a = _f32(a)
    col = np.ascontiguousarray(a.reshape(-1, 1))
    return gemm(col, np.ones((1, 1), np.float32), "nn", 1, iters).reshape(a.shape)


# ── the reference's per-MAC HIP arithmetic, compiled as host code ─────────

_hip = None


def hip_available() -> bool:
    return os.path.exists(HIP_PATH)


def hip() -> C.CDLL:
    """oracle/_ref/librac_hip_mac.so (built by build_ref_hip from rac_kernels.hip)."""
    global _hip
    if _hip is None:
        lib = C.CDLL(HIP_PATH, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        I, F, L = C.c_int, C.c_float, C.c_long
        lib.hipref_shiftadd_mul.argtypes = [F, F, I]
        lib.hipref_shiftadd_mul.restype = F
        lib.hipref_fma_cordic.argtypes = [F, F, F, I]
        lib.hipref_fma_cordic.restype = F
        lib.hipref_mac_batch.argtypes = [_fp, _fp, _fp, _fp, L, I, I]
        lib.hipref_rotate_n.argtypes = [_fp, _fp, _fp, L, I]
        lib.hipref_gemm.argtypes = [_fp, _fp, _fp, I, I, I, I, I, I]
        _hip = lib
    return _hip


def hip_mac(a, b, acc, iters: int, mode: int):
    """rac_fma_iters(a[i], b[i], acc[i], iters, mode) of rac_kernels.hip:202-218."""
    a, b, acc = _f32(a), _f32(b), _f32(acc)
    out = np.empty_like(a)
    hip().hipref_mac_batch(_p(a), _p(b), _p(acc), _p(out), a.size, iters, mode)
    return out


def hip_rotate_n(v, theta, iters: int):
    """rac_cordic_rotate_n of rac_kernels.hip:137-163 (no gain compensation)."""
    v, theta = _f32(v), _f32(theta)
    out = np.empty_like(v)
    hip().hipref_rotate_n(_p(v), _p(theta), _p(out), theta.size, iters)
    return out


def hip_gemm(A, B, layout: str = "nn", mode: int = 1, iters: int = 16):
    """Sequential-k GEMM over the reference's own rac_fma_iters."""
    A, B = _f32(A), _f32(B)
    lay = LAYOUTS[layout]
    K, M = A.shape if lay == 2 else A.shape[::-1]
    N = B.shape[0] if lay == 1 else B.shape[1]
    C_ = np.empty((M, N), np.float32)
    hip().hipref_gemm(_p(A), _p(B), _p(C_), M, N, K, lay, iters, mode)
    return C_


# ── the reference decoder bench's safetensors reader ───────────────────────

ST_PATH = os.path.join(HERE, "_ref", "libst_ref.so")
_st = None


def st_available() -> bool:
    return os.path.exists(ST_PATH)


class _StTensor(C.Structure):
    # bench/safetensors_reader.h: st_tensor (ST_MAX_NAME 256, ST_MAX_NDIM 8)
    _fields_ = [("name", C.c_char * 256), ("dtype", C.c_int), ("ndim", C.c_int),
                ("shape", C.c_int64 * 8), ("offset", C.c_size_t), ("nbytes", C.c_size_t)]


def ref_read_safetensors(path: str) -> dict:
    """Every tensor of a file through the reference reader (st_open, st_find,
    st_to_f32), as float32 arrays of the recorded shape."""
    global _st
    if _st is None:
        lib = C.CDLL(ST_PATH, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        lib.st_open.argtypes = [C.c_char_p, C.c_char_p]
        lib.st_open.restype = C.c_void_p
        lib.st_close.argtypes = [C.c_void_p]
        lib.st_find.argtypes = [C.c_void_p, C.c_char_p]
        lib.st_find.restype = C.POINTER(_StTensor)
        lib.st_numel.argtypes = [C.POINTER(_StTensor)]
        lib.st_numel.restype = C.c_size_t
        lib.st_to_f32.argtypes = [C.c_void_p, C.POINTER(_StTensor), _fp]
        lib.st_to_f32.restype = C.c_int
        _st = lib
    import json
    import struct
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        names = [k for k in json.loads(f.read(hlen)) if k != "__metadata__"]
    err = C.create_string_buffer(256)
    h = _st.st_open(path.encode(), err)
    if not h:
        raise RuntimeError(err.value.decode())
    try:
        out = {}
        for n in names:
            t = _st.st_find(h, n.encode())
            if not t:
                raise KeyError(n)
            shape = [t.contents.shape[i] for i in range(t.contents.ndim)]
            a = np.empty(int(_st.st_numel(t)), np.float32)
            if _st.st_to_f32(h, t, _p(a)) != 0:
                raise ValueError(f"{n}: dtype not convertible")
            out[n] = a.reshape(shape)
        return out
    finally:
        _st.st_close(h)


# ── reference-library front-ends ───────────────────────────────────────────

def ref_rotate_batch(v, theta):
    v, theta = _f32(v), _f32(theta)
    out = np.empty_like(v)
    ref().rac_rotate_batch(_p(v), _p(theta), _p(out), theta.size)
    return out


def ref_rotate_n_batch(v, theta, iters):
    v, theta = _f32(v), _f32(theta)
    out = np.empty_like(v)
    f = ref().rac_rotate_n
    for i in range(theta.size):
        r = f(Vec2(v[i, 0], v[i, 1]), float(theta[i]), iters)
        out[i] = (r.x, r.y)
    return out


def ref_project_n_batch(v, theta, iters):
    v, theta = _f32(v), _f32(theta)
    f = ref().rac_project_n
    return np.array([f(Vec2(v[i, 0], v[i, 1]), float(theta[i]), iters)
                     for i in range(theta.size)], np.float32)


def ref_rope_cache(max_seq, head_dim, base=10000.0):
    c = np.empty((max_seq, head_dim // 2), np.float32)
    s = np.empty_like(c)
    assert ref().rac_rope_cache(_p(c), _p(s), max_seq, head_dim, base) == 0
    return c, s


def ref_rope_apply(x, cos_tab, sin_tab):
    x = _f32(x).copy()
    b, h, s, hd = x.shape
    assert ref().rac_rope_apply(_p(x), _p(_f32(cos_tab)), _p(_f32(sin_tab)), b, h, s, hd, None) == 0
    return x


def ref_softmax(x):
    x = _f32(x)
    out = np.empty_like(x)
    ref().rac_softmax_batch(_p(x), _p(out), x.size // x.shape[-1], x.shape[-1])
    return out


def ref_rmsnorm(x, gamma=None, eps=1e-6):
    x = _f32(x)
    y = np.empty_like(x)
    g = _p(_f32(gamma)) if gamma is not None else None
    assert ref().rac_rmsnorm(_p(x), _p(y), g, eps, x.size // x.shape[-1], x.shape[-1], None) == 0
    return y


def ref_layernorm(x, gamma=None, beta=None, eps=1e-6):
    x = _f32(x)
    y = np.empty_like(x)
    g = _p(_f32(gamma)) if gamma is not None else None
    b = _p(_f32(beta)) if beta is not None else None
    assert ref().rac_layernorm(_p(x), _p(y), g, b, eps, x.size // x.shape[-1], x.shape[-1], None) == 0
    return y


def ref_sgemm(A, B):
    """lib/c HAL SGEMM (AVX2 path): the reference's CPU rac_matmul."""
    A, B = _f32(A), _f32(B)
    M, K = A.shape
    N = B.shape[1]
    C_ = np.empty((M, N), np.float32)
    assert ref().rac_hal_sgemm(_p(A), _p(B), _p(C_), M, N, K, 1.0, 0.0) == 0
    return C_


# ── tolerance helpers shared by the tests ──────────────────────────────────

def ulp_distance(a, b) -> np.ndarray:
    """Distance in units of float32 ordering (0 = bit equal)."""
    a = _f32(a).view(np.int32).astype(np.int64)
    b = _f32(b).view(np.int32).astype(np.int64)
    a = np.where(a < 0, np.int64(-2**31) - a, a)
    b = np.where(b < 0, np.int64(-2**31) - b, b)
    return np.abs(a - b)


def elementwise_ok(got, want, scale=None, max_ulp: int = 2) -> np.ndarray:
    """Elementwise bar: <= max_ulp ulps, or |diff| <= max_ulp * ulp(max(1, |scale|))."""
    got, want = _f32(got), _f32(want)
    if scale is None:
        scale = np.maximum(np.abs(want), 1.0)
    floor = max_ulp * np.spacing(np.maximum(np.abs(_f32(scale)), np.float32(1.0)))
    return (ulp_distance(got, want) <= max_ulp) | (np.abs(got - want) <= floor)


def max_rel_err(got, want) -> float:
    """Reduction bar metric: max |got-want| / max(|want|, 1e-3 * rms(want))."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    if want.size == 0:
        return 0.0
    rms = np.sqrt(np.mean(want * want)) if want.size else 0.0
    den = np.maximum(np.abs(want), 1e-3 * rms + 1e-30)
    return float(np.max(np.abs(got - want) / den))


def reduction_ok(got, want, exact=None, tol: float = 1e-4) -> bool:
    """Reduction bar: max_rel_err(got, want) <= tol.  Where the reference's own
    float32 rounding already exceeds tol against the float64 `exact` result
    (LayerNorm's x - mean cancellation does), the bar is instead: no farther
    from exact than 1.5x the reference, and normwise within tol/10 of it."""
    if max_rel_err(got, want) <= tol:
        return True
    if exact is None:
        return False
    want = np.asarray(want, np.float64)
    rms = float(np.sqrt(np.mean(want * want))) or 1.0
    normwise = float(np.abs(np.asarray(got, np.float64) - want).max()) / rms
    return normwise <= tol / 10 and max_rel_err(got, exact) <= 1.5 * max_rel_err(want, exact)
