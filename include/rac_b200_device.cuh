/* rac_b200_device.cuh -- header-only device API: the RAC primitives for use
 * inside your own CUDA kernels (sm_100a).
 *
 * Each function computes, for one element, exactly the bits the library's
 * batch entry points compute for it (they run the same device code):
 *
 *   rac_dev_rotate(v, th)            rac_rotate / rac_rotate_batch
 *                                    (RAC_K_INV pre-scale, 16 iterations;
 *                                    ref lib/c/rac_cpu.c:136-139, 344-349)
 *   rac_dev_rotate_n(v, th, n)       rac_rotate_precision / rac_rotate_batch_n
 *                                    (1/K(n) pre-scale, n clamped to [4, 24];
 *                                    ref lib/c/rac_cpu.c:275-280)
 *   rac_dev_project_n(v, th, n)      rac_project_precision / rac_project_batch_n
 *                                    (ref lib/c/rac_cpu.c:282-288)
 *   rac_dev_sincos(th, &s, &c)       rac_sincos (ref lib/c/rac_cpu.c:322-328)
 *   rac_dev_fma_cordic(acc, a, b, n) one CORDIC MAC of rac_matmul: acc +
 *                                    (x_n(a folded by b's sign) / K(n)) * |b|,
 *                                    n clamped to [1, 24]
 *                                    (ref rac_torch/rac_kernels.hip:139-185)
 *
 * theta must be finite: the reference's wrap loop never ends for |theta| >=
 * 2^25 or inf; here it stops after 2^20 steps (the batch entry points report
 * that as RAC_ERR_DEVICE; these functions return an unspecified value).
 *
 * Compile with nvcc -gencode arch=compute_100a,code=sm_100a and
 * -I<this directory>.
 *
 * Location: this header includes the library's internal device code
 * (rac_b200/csrc/rac_device.cuh) by its path relative to this directory, so
 * it compiles only from inside the source tree (or an install that keeps
 * include/ and rac_b200/csrc/ side by side).  Only the rac_dev_* functions
 * below are the public API; the racb:: names they use are internal and may
 * change between versions.
 */
#pragma once

#include <cuda_runtime.h>

#include "../rac_b200/csrc/rac_device.cuh"

__device__ __forceinline__ float2 rac_dev_rotate(float2 v, float theta) {
    float x, y;
    racb::cordic_rotate_scaled<racb::kDefaultIters>(x, y, v.x, v.y, racb::kKInv, theta);
    return make_float2(x, y);
}

__device__ __forceinline__ float2 rac_dev_rotate_n(float2 v, float theta, int iters) {
    iters = iters < 4 ? 4 : (iters > racb::kMaxIters ? racb::kMaxIters : iters);
    const float k = racb::k_inv_of(iters);
    float x = __fmul_rn(v.x, k), y = __fmul_rn(v.y, k);
    racb::cordic_rotate_rt(x, y, theta, iters);
    return make_float2(x, y);
}

__device__ __forceinline__ float rac_dev_project_n(float2 v, float theta, int iters) {
    iters = iters < 4 ? 4 : (iters > racb::kMaxIters ? racb::kMaxIters : iters);
    float c = racb::k_inv_of(iters), s = 0.0f;
    racb::cordic_rotate_rt(c, s, theta, iters);
    return __fmaf_rn(v.x, c, __fmul_rn(v.y, s));
}

__device__ __forceinline__ void rac_dev_sincos(float theta, float* s, float* c) {
    float cc, ss;
    racb::cordic_rotate_scaled<racb::kDefaultIters>(cc, ss, 1.0f, 0.0f, racb::kKInv, theta);
    *s = ss;
    *c = cc;
}

__device__ __forceinline__ float rac_dev_fma_cordic(float acc, float a, float b, int iters) {
    iters = iters < 1 ? 1 : (iters > racb::kMaxIters ? racb::kMaxIters : iters);
    const unsigned sgn = __float_as_uint(b) & 0x80000000u;
    const float mag = __uint_as_float(__float_as_uint(b) & 0x7FFFFFFFu);
    const float sa = __uint_as_float(__float_as_uint(a) ^ sgn);
    float x = sa, y = sa;                          // iteration 0: (sa, 0) -> (sa, sa)
    for (int t = 1; t < iters; ++t) {
        const float cf = racb::gemm_coef(t);
        const float xn = __fmaf_rn(-cf, y, x);
        y = __fmaf_rn(cf, x, y);
        x = xn;
    }
    return __fmaf_rn(__fmul_rn(x, racb::k_inv_of(iters)), mag, acc);
}
