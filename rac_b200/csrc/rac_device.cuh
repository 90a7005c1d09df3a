// rac_device.cuh -- device-side CORDIC primitives for sm_100a.
//
// Semantics follow the reference CPU library lib/c/rac_cpu.c (the parity
// target) and the GPU GEMM of rac_torch/rac_kernels.hip; every rounding step
// is written with an explicit __f*_rn intrinsic so that nvcc cannot contract
// or reassociate it.  Cited lines are inside the Pinnacle-Quantum-Group/RAC
// project.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace racb {

// RAC_PI, RAC_K_INV, RAC_ITERS: lib/c/rac_cpu.h:39-42.
constexpr float kPi = 3.14159265358979f;
constexpr float kKInv = 0.60725f;
constexpr int kDefaultIters = 16;
constexpr int kMaxIters = 24;
// Upper bound on the (-pi, pi] wrap loop of _cordic_rotate (lib/c/rac_cpu.c:93-94).
// The reference loops forever when theta - 2*pi == theta (|theta| >= 2^25 or
// inf); a GPU thread must not, so the loop stops here and flags the launch.
constexpr int kWrapLimit = 1 << 20;

// atan(2^-i) table, i = 0..23 (lib/c/rac_cpu.c:20-25 + :37-40; identical in
// rac_torch/rac_kernels.hip:32-39), for runtime-indexed loops.
__device__ __constant__ static const float kAtanTab[24] = {
    0.78539816f, 0.46364761f, 0.24497866f, 0.12435499f,
    0.06241881f, 0.03123983f, 0.01562373f, 0.00781234f,
    0.00390623f, 0.00195312f, 0.00097656f, 0.00048828f,
    0.00024414f, 0.00012207f, 0.00006104f, 0.00003052f,
    0.00001526f, 0.00000763f, 0.00000381f, 0.00000191f,
    0.00000095f, 0.00000048f, 0.00000024f, 0.00000012f,
};

// The same table as a constexpr function, so that unrolled device loops fold
// table entries to immediates (the __constant__ copy serves runtime indices).
__host__ __device__ constexpr float atan_entry(int i) {
    constexpr float t[24] = {
        0.78539816f, 0.46364761f, 0.24497866f, 0.12435499f,
        0.06241881f, 0.03123983f, 0.01562373f, 0.00781234f,
        0.00390623f, 0.00195312f, 0.00097656f, 0.00048828f,
        0.00024414f, 0.00012207f, 0.00006104f, 0.00003052f,
        0.00001526f, 0.00000763f, 0.00000381f, 0.00000191f,
        0.00000095f, 0.00000048f, 0.00000024f, 0.00000012f,
    };
    return t[i];
}

// CORDIC gain K(n), n = 0..24 (lib/c/rac_cpu.c:44-52, rac_kernels.hip:42-50).
__host__ __device__ constexpr float k_entry(int n) {
    constexpr float t[25] = {
        1.00000000f, 1.41421356f, 1.58113883f, 1.62979295f,
        1.64248460f, 1.64568447f, 1.64648404f, 1.64668388f,
        1.64673383f, 1.64674632f, 1.64674944f, 1.64675022f,
        1.64675042f, 1.64675047f, 1.64675048f, 1.64675049f,
        1.64675049f, 1.64675049f, 1.64675049f, 1.64675049f,
        1.64675049f, 1.64675049f, 1.64675049f, 1.64675049f,
        1.64675049f,
    };
    return t[n];
}

// Direction sequence of the GEMM MAC.  In rac_fma_cordic
// (rac_kernels.hip:176-185) b is encoded as angle 0 or pi; pi folds to 0 with
// a negated vector (:144-150), so the residual angle always starts at +0 and
// d_i = sign(angle_i) follows from the atan table alone:
//   angle_0 = 0, d_i = (angle_i >= 0) ? +1 : -1, angle_{i+1} = angle_i - d_i*atan_i
// evaluated in float32.  A host test recomputes the recursion and checks it
// against rac_b200_cordic_gemm_directions() (exported by the shim).
__host__ __device__ constexpr int gemm_dir(int i) {
    constexpr int t[24] = {
        +1, -1, -1, -1, +1, -1, +1, +1, -1, -1, -1, -1,
        +1, +1, -1, -1, +1, +1, -1, -1, +1, -1, -1, +1,
    };
    return t[i];
}

// 2^-i (exact).
__host__ __device__ constexpr float pow2neg(int i) {
    float s = 1.0f;
    for (int t = 0; t < i; ++t) s *= 0.5f;
    return s;
}

// d_i * 2^-i, the micro-rotation coefficient of iteration i of the GEMM MAC.
__host__ __device__ constexpr float gemm_coef(int i) {
    return gemm_dir(i) > 0 ? pow2neg(i) : -pow2neg(i);
}

// One CORDIC MAC of rac_fma_cordic (rac_kernels.hip:176-185) with the fold
// already applied: the vector entering the iterations is (sa, 0) where
// sa = a with b's sign bit xor-ed in (the fold negates it when b < 0).
// Iteration i is x' = x - c_i*y, y' = y + c_i*x with c_i = d_i*2^-i, one
// rounding each (the product c_i*y is exact for normal values).  Only x of
// the last iteration is used.  Returns x_n (before the 1/K(n) compensation).
//
// Instruction economy, bit-identical for normal sa:
//  - iteration 0 (scale 1, y = 0) maps (sa, 0) to (sa, sa): a copy;
//  - iteration 1 (d_1 = -1) gives x = fl(1.5 sa) and y = sa/2 exactly, so y
//    is carried from here on as ys = 2y (scaling by 2 commutes with
//    rounding): ys = sa costs nothing, and later iterations use
//    x' = x - (c_i/2)*ys, ys' = ys + (2 c_i)*x, still one rounding each.
// That is 2n - 3 FFMAs for n micro-rotations (plus the LOP3 fold, the 1/K(n)
// FMUL and the accumulating FFMA: 2n - 1 instructions per MAC).
template <int ITERS>
__device__ __forceinline__ float gemm_cordic_x(float sa) {
    static_assert(gemm_dir(1) < 0, "the y = sa/2 shortcut needs d_1 = -1");
    if constexpr (ITERS <= 1) {
        return sa;
    } else {
        float x = __fmaf_rn(-gemm_coef(1), sa, sa);       // iteration 1
        float ys = sa;                                     // 2 * y_2
#pragma unroll
        for (int t = 2; t < ITERS; ++t) {
            const float c = gemm_coef(t);
            if (t == ITERS - 1) {
                x = __fmaf_rn(-0.5f * c, ys, x);
            } else {
                const float xn = __fmaf_rn(-0.5f * c, ys, x);
                ys = __fmaf_rn(2.0f * c, x, ys);
                x = xn;
            }
        }
        return x;
    }
}

// gemm_cordic_x for two independent operands at once: the same micro-
// rotations as packed FFMA2 (each half one fused multiply-add, rounded once:
// the bits of the scalar form).
template <int ITERS>
__device__ __forceinline__ float2 gemm_cordic_x2(float2 sa) {
    if constexpr (ITERS <= 1) {
        return sa;
    } else {
        float2 x = __ffma2_rn(make_float2(-gemm_coef(1), -gemm_coef(1)), sa, sa);
        float2 ys = sa;
#pragma unroll
        for (int t = 2; t < ITERS; ++t) {
            const float c = gemm_coef(t);
            const float2 c1 = make_float2(-0.5f * c, -0.5f * c), c2 = make_float2(2.0f * c, 2.0f * c);
            if (t == ITERS - 1) {
                x = __ffma2_rn(c1, ys, x);
            } else {
                const float2 xn = __ffma2_rn(c1, ys, x);
                ys = __ffma2_rn(c2, x, ys);
                x = xn;
            }
        }
        return x;
    }
}

// Runtime-iteration variant (any n in [1, 24]); coefficients come from a
// kernel-argument table.
__device__ __forceinline__ float gemm_cordic_x_rt(float sa, int iters,
                                                   const float* coef) {
    float x = sa, y = sa;
    for (int t = 1; t < iters; ++t) {
        const float c = coef[t];
        const float xn = __fmaf_rn(-c, y, x);
        y = __fmaf_rn(c, x, y);
        x = xn;
    }
    return x;
}

// Bit pattern of 2^-i, i = 0..126.
__host__ __device__ constexpr unsigned pow2neg_bits(int i) { return (unsigned)(127 - i) << 23; }

// atan_i * 2^i (exact: a power-of-two scaling of a normal float).
__host__ __device__ constexpr float atan_scaled(int i) {
    float a = atan_entry(i);
    for (int k = 0; k < i; ++k) a *= 2.0f;
    return a;
}

// _cordic_rotate of lib/c/rac_cpu.c:90-118 on (vx * kinv, vy * kinv): wrap
// theta to (-pi, pi], fold into [-pi/2, pi/2] by negating (x, y), then ITERS
// micro-rotations whose direction d_i = (angle_i >= 0) ? +1 : -1 is the sign
// of the residual angle.  Returns false when the wrap loop hit kWrapLimit.
//
// Same roundings as the reference, fewer instructions:
//  * the wrap loops run only when |theta| >= pi (NaN skips them, as there);
//  * the fold's negation of (x, y) is folded into the scale: vx * -kinv is
//    -(vx * kinv) exactly;
//  * the fold's theta -/+ pi is theta + c with c = -copysign(pi, theta),
//    which is the same rounded value; without a fold c = +0, which maps -0
//    to +0 and leaves every other angle unchanged, so that the sign bit of
//    the angle is the comparison angle >= 0 from iteration 0 on;
//  * a NaN angle gives d_i = -1 in the reference (the comparison is false)
//    and is replaced by -inf (fmaxf(NaN, -inf) = -inf), which stays -inf.
// Each iteration is then four instructions, one on the ALU pipe and three on
// the FMA pipe:
//   ds = (angle & sign) | bits(2^-i)          = d_i * 2^-i   (one LOP3)
//   x, y updated with ds                       (two FFMA)
//   angle - d_i*atan_i = fma(-ds, atan_i*2^i, angle): ds * (atan_i*2^i)
//   equals d_i*atan_i exactly (power-of-two scalings), and the FMA rounds
//   once, as the subtraction of the exact product does.  (one FFMA)
// For i >= 1 the angle is a rounded difference with a nonzero table entry,
// so it is never -0 either.
//
// sign_mask must be 0x80000000.  A kernel that passes it in as a launch
// argument keeps it in a register, so each direction is one LOP3
// ((angle & mask) | imm); with the literal default the compiler folds the
// mask and needs two.
template <int ITERS>
__device__ __forceinline__ bool cordic_rotate_scaled(float& xr, float& yr, float vx, float vy,
                                                     float kinv, float theta,
                                                     unsigned sign_mask = 0x80000000u) {
    bool ok = true;
    if (fabsf(theta) >= kPi) {
        const float TAU = 2.0f * kPi;
        int w = 0;
        while (theta > kPi) { theta = __fsub_rn(theta, TAU); if (++w >= kWrapLimit) { ok = false; break; } }
        while (theta <= -kPi) { theta = __fadd_rn(theta, TAU); if (++w >= kWrapLimit) { ok = false; break; } }
    }
    const bool fold = fabsf(theta) > kPi * 0.5f;
    const float c = fold ? __uint_as_float((~__float_as_uint(theta) & sign_mask) | __float_as_uint(kPi))
                         : 0.0f;
    float angle = fmaxf(__fadd_rn(theta, c), -INFINITY);
    const float ks = fold ? -kinv : kinv;
    float x = __fmul_rn(vx, ks), y = __fmul_rn(vy, ks);
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        unsigned dsb;
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;"           // (angle & sign_mask) | bits(2^-i)
            : "=r"(dsb) : "r"(__float_as_uint(angle)), "r"(sign_mask), "r"(pow2neg_bits(i)));
        const float ds = __uint_as_float(dsb);
        const float xn = __fmaf_rn(-ds, y, x);
        y = __fmaf_rn(ds, x, y);
        x = xn;
        if (i + 1 < ITERS)
            angle = __fmaf_rn(-ds, atan_scaled(i), angle);  // angle - d_i*atan_i, one rounding
    }
    xr = x; yr = y;
    return ok;
}

// Two independent rotations at once: the prologue per vector as above, then
// the micro-rotations of both vectors as packed pairs -- the x, y and angle
// updates of the two vectors are three FFMA2 (two FMAs each, each rounded
// once: the bits of the scalar form) instead of six FFMA, with the two
// directions from one LOP3 each.
template <int ITERS>
__device__ __forceinline__ bool cordic_rotate_scaled_x2(float& xa, float& ya, float& xb, float& yb,
                                                        float vxa, float vya, float vxb, float vyb,
                                                        float kinv, float tha, float thb,
                                                        unsigned sign_mask = 0x80000000u) {
    bool ok = true;
    float ang[2], px[2], py[2];
    const float th2[2] = {tha, thb}, vx2[2] = {vxa, vxb}, vy2[2] = {vya, vyb};
#pragma unroll
    for (int v = 0; v < 2; ++v) {
        float theta = th2[v];
        if (fabsf(theta) >= kPi) {
            const float TAU = 2.0f * kPi;
            int w = 0;
            while (theta > kPi) { theta = __fsub_rn(theta, TAU); if (++w >= kWrapLimit) { ok = false; break; } }
            while (theta <= -kPi) { theta = __fadd_rn(theta, TAU); if (++w >= kWrapLimit) { ok = false; break; } }
        }
        const bool fold = fabsf(theta) > kPi * 0.5f;
        const float c = fold ? __uint_as_float((~__float_as_uint(theta) & sign_mask) | __float_as_uint(kPi))
                             : 0.0f;
        ang[v] = fmaxf(__fadd_rn(theta, c), -INFINITY);
        const float ks = fold ? -kinv : kinv;
        px[v] = __fmul_rn(vx2[v], ks);
        py[v] = __fmul_rn(vy2[v], ks);
    }
    float2 X = make_float2(px[0], px[1]), Y = make_float2(py[0], py[1]), A = make_float2(ang[0], ang[1]);
#pragma unroll
    for (int i = 0; i < ITERS; ++i) {
        unsigned da, db;
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(da) : "r"(__float_as_uint(A.x)), "r"(sign_mask), "r"(pow2neg_bits(i)));
        asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(db) : "r"(__float_as_uint(A.y)), "r"(sign_mask), "r"(pow2neg_bits(i)));
        const float2 DS = make_float2(__uint_as_float(da), __uint_as_float(db));
        const float2 NDS = make_float2(-DS.x, -DS.y);
        const float2 Xn = __ffma2_rn(NDS, Y, X);
        Y = __ffma2_rn(DS, X, Y);
        X = Xn;
        if (i + 1 < ITERS) A = __ffma2_rn(NDS, make_float2(atan_scaled(i), atan_scaled(i)), A);
    }
    xa = X.x; xb = X.y; ya = Y.x; yb = Y.y;
    return ok;
}

// The same rotation of an already scaled (x, y).
template <int ITERS>
__device__ __forceinline__ bool cordic_rotate(float& xr, float& yr, float theta,
                                              unsigned sign_mask = 0x80000000u) {
    return cordic_rotate_scaled<ITERS>(xr, yr, xr, yr, 1.0f, theta, sign_mask);
}

// Runtime-iteration version of the same rotation (iters in [1, 24]).
__device__ __forceinline__ bool cordic_rotate_rt(float& xr, float& yr, float theta, int iters) {
    const float TAU = 2.0f * kPi;
    bool ok = true;
    int w = 0;
    while (theta > kPi) { theta = __fsub_rn(theta, TAU); if (++w >= kWrapLimit) { ok = false; break; } }
    while (theta <= -kPi) { theta = __fadd_rn(theta, TAU); if (++w >= kWrapLimit) { ok = false; break; } }
    float x = xr, y = yr;
    if (theta > kPi * 0.5f) {
        x = -x; y = -y; theta = __fsub_rn(theta, kPi);
    } else if (theta < -kPi * 0.5f) {
        x = -x; y = -y; theta = __fadd_rn(theta, kPi);
    }
    float angle = theta, s = 1.0f;
    for (int i = 0; i < iters; ++i) {
        const float d = (angle >= 0.0f) ? 1.0f : -1.0f;
        const float ds = d * s;                     // exact
        const float xn = __fmaf_rn(-ds, y, x);
        y = __fmaf_rn(ds, x, y);
        x = xn;
        angle = __fsub_rn(angle, d * kAtanTab[i]);  // d * atan is exact
        s *= 0.5f;
    }
    xr = x; yr = y;
    return ok;
}

// rac_shiftadd_mul (rac_torch/rac_kernels.hip:84-122): a * b from the top
// `iters` bits of b's 24-bit mantissa by integer shift-and-add on the
// INT pipe (no FP multiplier), truncated into fp32, sub/super-normal results
// flushed to 0.  The 48-bit product is kept as two 32-bit words.
__device__ __forceinline__ float shiftadd_mul(float a, float b, int iters) {
    if (a == 0.0f || b == 0.0f) return 0.0f;
    const uint32_t ai = __float_as_uint(a), bi = __float_as_uint(b);
    const uint32_t sign = (ai ^ bi) & 0x80000000u;
    const int exp_a = (int)((ai >> 23) & 0xFFu) - 127;
    const int exp_b = (int)((bi >> 23) & 0xFFu) - 127;
    const uint32_t ma = 0x00800000u | (ai & 0x007FFFFFu);
    const uint32_t mb = 0x00800000u | (bi & 0x007FFFFFu);
    const int lim = iters < 1 ? 1 : (iters > 24 ? 24 : iters);
    unsigned long long prod = 0ull;
    for (int i = 0; i < lim; ++i) {
        const int sh = 23 - i;
        const unsigned long long term = ((unsigned long long)ma) << sh;
        prod += ((mb >> sh) & 1u) ? term : 0ull;
    }
    if (prod == 0ull) return 0.0f;
    const int top = 63 - __clzll((long long)prod);
    const int shift_r = top - 23;
    uint32_t mantissa;
    if (shift_r > 0) mantissa = (uint32_t)(prod >> shift_r) & 0x007FFFFFu;
    else if (shift_r < 0) mantissa = (uint32_t)(prod << -shift_r) & 0x007FFFFFu;
    else mantissa = (uint32_t)prod & 0x007FFFFFu;
    const int rexp = exp_a + exp_b + (top - 46) + 127;
    if (rexp <= 0 || rexp >= 0xFF) return 0.0f;
    return __uint_as_float(sign | ((uint32_t)(rexp & 0xFF) << 23) | mantissa);
}

// 1/K(n) in float, as both reference libraries compute it at run time
// (lib/c/rac_cpu.c:277, rac_kernels.hip:182).
__host__ __device__ inline float k_inv_of(int iters) {
    return 1.0f / k_entry(iters);
}

}  // namespace racb
