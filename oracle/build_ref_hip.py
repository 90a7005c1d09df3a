"""Compiles the reference's per-MAC device arithmetic (rac_torch/rac_kernels.hip)
as host C++ into ``oracle/_ref/librac_hip_mac.so`` -- TEST INFRASTRUCTURE ONLY.

The reference's CORDIC and SHIFTADD GEMMs exist only as HIP kernels, which
cannot be built here (no hipcc).  Their arithmetic, though, is three
self-contained ``__device__`` functions plus two constant tables:

* ``rac_shiftadd_mul``   rac_kernels.hip:84-122   (integer shift-add product)
* ``rac_cordic_rotate_n`` rac_kernels.hip:137-163 (n micro-rotations)
* ``rac_fma_cordic``      rac_kernels.hip:176-185 (the CORDIC-mode MAC)
* ``rac_fma_iters``       rac_kernels.hip:202-218 (the per-MAC mode dispatch)
* ``rac_atan_table`` / ``rac_k_table`` rac_kernels.hip:32-50

This recipe reads those definitions out of the reference file by name (brace
matching, so the cited ranges need not be hard-coded), prepends a small shim
that maps the handful of CUDA/HIP spellings they use onto host C++
(``__float_as_uint`` -> memcpy bit cast, ``__clzll`` -> ``__builtin_clzll``,
``__constant__`` -> ``static const``), appends a sequential-k GEMM driver that
calls ``rac_fma_iters`` per MAC -- the accumulation order of every reference
GEMM tier -- and pipes the translation unit to g++ on standard input.  No
reference source is written to disk; only the compiled library lands in
``oracle/_ref/`` (git-ignored).

The library is built with -ffp-contract=fast, hipcc's default: the
micro-rotation ``x - d*y*scale`` then rounds once (a fused multiply-add), as
the HIP build of the reference does.  For operands in the normal range the
contraction changes nothing (d*y*2^-i and d*atan_i are exact products); it
matters only where d*y*2^-i falls below the normal range (|a| near 2^-126),
where the unfused form would round that product first.

    python -m oracle.build_ref_hip [REFERENCE_ROOT]
"""
from __future__ import annotations

import os
import re
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref", "librac_hip_mac.so")

_SHIM = r"""
#include <cmath>
#include <cstring>
#include <cstdint>
#define __device__
#define __forceinline__ inline
#define __constant__ static const
struct float2 { float x, y; };
static inline float2 make_float2(float x, float y) { float2 r; r.x = x; r.y = y; return r; }
static inline unsigned int __float_as_uint(float f) { unsigned int u; std::memcpy(&u, &f, 4); return u; }
static inline float __uint_as_float(unsigned int u) { float f; std::memcpy(&f, &u, 4); return f; }
static inline int __clzll(unsigned long long v) { return v ? __builtin_clzll(v) : 64; }
#define RAC_MODE_FAST     0
#define RAC_MODE_CORDIC   1
#define RAC_MODE_SHIFTADD 2
"""

_DRIVER = r"""
extern "C" {
float hipref_shiftadd_mul(float a, float b, int iters) { return rac_shiftadd_mul(a, b, iters); }
float hipref_fma_cordic(float a, float b, float acc, int iters) { return rac_fma_cordic(a, b, acc, iters); }
float hipref_fma_iters(float a, float b, float acc, int iters, int mode) {
    return rac_fma_iters(a, b, acc, iters, mode);
}
void hipref_mac_batch(const float *a, const float *b, const float *acc, float *out, long n,
                      int iters, int mode) {
    for (long i = 0; i < n; i++) out[i] = rac_fma_iters(a[i], b[i], acc[i], iters, mode);
}
void hipref_rotate_n(const float *v, const float *theta, float *out, long n, int iters) {
    for (long i = 0; i < n; i++) {
        float2 r = rac_cordic_rotate_n(make_float2(v[2 * i], v[2 * i + 1]), theta[i], iters);
        out[2 * i] = r.x; out[2 * i + 1] = r.y;
    }
}
/* C[M,N] = sum_k mac(A[m,k], B[k,n]) in k order; layout 0 NN (A[M,K], B[K,N]),
   1 NT (B[N,K]), 2 TN (A[K,M]). */
void hipref_gemm(const float *A, const float *B, float *C, int M, int N, int K,
                 int layout, int iters, int mode) {
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; m++)
        for (int n = 0; n < N; n++) {
            float acc = 0.0f;
            for (int k = 0; k < K; k++) {
                float a = layout == 2 ? A[(long)k * M + m] : A[(long)m * K + k];
                float b = layout == 1 ? B[(long)n * K + k] : B[(long)k * N + n];
                acc = rac_fma_iters(a, b, acc, iters, mode);
            }
            C[(long)m * N + n] = acc;
        }
}
}
"""

# Definitions taken from the reference file, in dependency order.
_NAMES = ["rac_atan_table", "rac_k_table", "rac_shiftadd_mul", "rac_cordic_rotate_n",
          "rac_fma_cordic", "rac_fma_iters"]


def _extract(lines: list[str], name: str) -> str:
    """The top-level definition of `name`: from the line that names it (plus a
    preceding qualifier-only line such as ``__device__ __forceinline__``) to the
    line that closes its outermost brace."""
    pat = re.compile(r"^[A-Za-z_].*\b" + re.escape(name) + r"\s*[\(\[]")
    for i, ln in enumerate(lines):
        if pat.match(ln):
            start = i
            if i > 0 and re.fullmatch(r"\s*(__device__|__forceinline__|\s)+\s*", lines[i - 1]):
                start = i - 1
            depth, seen = 0, False
            for j in range(i, len(lines)):
                depth += lines[j].count("{") - lines[j].count("}")
                seen = seen or "{" in lines[j]
                if seen and depth == 0:
                    return "".join(lines[start:j + 1])
            break
    raise RuntimeError(f"definition of {name} not found in rac_kernels.hip")


def default_root() -> str:
    """RAC_REF_ROOT, else a checkout named ``reference`` beside this repository."""
    return os.environ.get("RAC_REF_ROOT") or os.path.join(
        os.path.dirname(os.path.dirname(HERE)), "reference")


def build(ref_root: str | None = None) -> str | None:
    src = os.path.join(ref_root or default_root(), "rac_torch", "rac_kernels.hip")
    if not os.path.exists(src):
        return None
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= max(os.path.getmtime(src),
                                                             os.path.getmtime(__file__)):
        return OUT
    with open(src) as f:
        lines = f.readlines()
    tu = _SHIM + "".join(f'#line 1 "{n}"\n' + _extract(lines, n) + "\n" for n in _NAMES) + _DRIVER
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    cmd = ["g++", "-O2", "-mfma", "-ffp-contract=fast", "-fopenmp", "-fPIC", "-shared",
           "-x", "c++", "-", "-o", OUT + ".tmp"]
    r = subprocess.run(cmd, input=tu, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"g++ failed on the extracted reference MAC:\n{r.stderr}")
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(*(sys.argv[1:2] or [])))
