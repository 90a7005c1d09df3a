/*
 * rac_oracle.c -- CPU restatement of the RAC rotation-accumulate hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * kernels in rac_b200/csrc.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py load it.  The product
 * path never calls it and has no CPU fallback.
 *
 * Every function restates one reference routine; the reference file:line is
 * given beside it (paths inside the Pinnacle-Quantum-Group/RAC project).
 * The restatement is compiled with -ffp-contract=off so that every rounding
 * step is the one written in the source: that is the contract the GPU
 * kernels follow with explicit __fmaf_rn/__fmul_rn/__fadd_rn placement, and
 * the GPU results are checked bit-for-bit against this file where the
 * reduction order allows it.
 *
 * Pinning: tests/test_oracle.py checks this restatement against the
 * reference's own lib/c built from its sources (oracle/_ref/librac_ref.so,
 * recipe oracle/Makefile) and against the known-answer cases of
 * lib/c/test_rac_lib_bvt.c and lib/c/test_rac_lib_dvt.c.
 *
 * All symbols carry the orc_ prefix so the library can share a process with
 * both the reference library and the product shim (the three export
 * same-named rac_* symbols with different signatures otherwise).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_PI       3.14159265358979f  /* lib/c/rac_cpu.h:42 (RAC_PI)        */
#define ORC_K_INV    0.60725f           /* lib/c/rac_cpu.h:39 (RAC_K_INV)     */
#define ORC_ITERS    16                 /* lib/c/rac_cpu.h:41 (RAC_ITERS)     */

/* atan(2^-i), i = 0..23: lib/c/rac_cpu.c:20-25 (first 16) and :37-40 (ext);
 * identical values in rac_torch/rac_kernels.hip:32-39. */
static const float orc_atan[24] = {
    0.78539816f, 0.46364761f, 0.24497866f, 0.12435499f,
    0.06241881f, 0.03123983f, 0.01562373f, 0.00781234f,
    0.00390623f, 0.00195312f, 0.00097656f, 0.00048828f,
    0.00024414f, 0.00012207f, 0.00006104f, 0.00003052f,
    0.00001526f, 0.00000763f, 0.00000381f, 0.00000191f,
    0.00000095f, 0.00000048f, 0.00000024f, 0.00000012f,
};

/* CORDIC gain K(n), n = 0..24: lib/c/rac_cpu.c:44-52, rac_kernels.hip:42-50. */
static const float orc_k[25] = {
    1.00000000f, 1.41421356f, 1.58113883f, 1.62979295f,
    1.64248460f, 1.64568447f, 1.64648404f, 1.64668388f,
    1.64673383f, 1.64674632f, 1.64674944f, 1.64675022f,
    1.64675042f, 1.64675047f, 1.64675048f, 1.64675049f,
    1.64675049f, 1.64675049f, 1.64675049f, 1.64675049f,
    1.64675049f, 1.64675049f, 1.64675049f, 1.64675049f,
    1.64675049f,
};

const float *orc_atan_table(void) { return orc_atan; }
const float *orc_k_table(void) { return orc_k; }

/* lib/c/rac_cpu.c:54-58 -- iteration clamp of the CPU library. */
int orc_clamp_iters_cpu(int n) { return n < 4 ? 4 : (n > 24 ? 24 : n); }
/* rac_torch/rac_kernels.hip:816-820 -- clamp of the GPU GEMM launchers. */
int orc_clamp_iters_gemm(int n) { return n < 1 ? 1 : (n > 24 ? 24 : n); }

/* lib/c/rac_cpu.c:90-118 (_cordic_rotate): wrap to (-pi, pi], fold into
 * [-pi/2, pi/2] by negating the vector, then `iters` micro-rotations with
 * the direction taken from the sign of the residual angle. */
static void orc_cordic_rotate(float *px, float *py, float theta, int iters) {
    const float TAU = 2.0f * ORC_PI;
    while (theta > ORC_PI) theta -= TAU;
    while (theta <= -ORC_PI) theta += TAU;
    float x = *px, y = *py;
    if (theta > ORC_PI * 0.5f) {
        x = -x; y = -y; theta -= ORC_PI;
    } else if (theta < -ORC_PI * 0.5f) {
        x = -x; y = -y; theta += ORC_PI;
    }
    float angle = theta, scale = 1.0f;
    for (int i = 0; i < iters; i++) {
        float d = (angle >= 0.0f) ? 1.0f : -1.0f;
        float xn = x - d * y * scale;   /* d*y*scale is exact: one rounding */
        float yn = y + d * x * scale;
        angle -= d * orc_atan[i];
        x = xn; y = yn;
        scale *= 0.5f;
    }
    *px = x; *py = y;
}

/* lib/c/rac_cpu.c:136-139 (rac_rotate): pre-scale by the literal RAC_K_INV,
 * then 16 iterations.  lib/c/rac_cpu.c:275-280 (rac_rotate_n): pre-scale by
 * 1/K(n) with n clamped to [4, 24].  `literal_kinv` selects the former. */
void orc_rotate(float vx, float vy, float theta, int iters, int literal_kinv,
                float *ox, float *oy) {
    float k_inv;
    if (literal_kinv) { k_inv = ORC_K_INV; iters = ORC_ITERS; }
    else { iters = orc_clamp_iters_cpu(iters); k_inv = 1.0f / orc_k[iters]; }
    float x = vx * k_inv, y = vy * k_inv;
    orc_cordic_rotate(&x, &y, theta, iters);
    *ox = x; *oy = y;
}

/* lib/c/rac_cpu.c:344-349 (rac_rotate_batch) when literal_kinv = 1, or a
 * batch of rac_rotate_n (lib/c/rac_cpu.c:275-280) otherwise.
 * v and out are interleaved float2 arrays. */
void orc_rotate_batch(const float *v, const float *theta, float *out,
                      long n, int iters, int literal_kinv) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; i++)
        orc_rotate(v[2 * i], v[2 * i + 1], theta[i], iters, literal_kinv,
                   &out[2 * i], &out[2 * i + 1]);
}

/* lib/c/rac_cpu.c:282-288 (rac_project_n): rotate (1/K(n), 0) by theta,
 * then fmaf(v.x, c, v.y * s). */
float orc_project_n(float vx, float vy, float theta, int iters) {
    iters = orc_clamp_iters_cpu(iters);
    float x = 1.0f / orc_k[iters], y = 0.0f;
    orc_cordic_rotate(&x, &y, theta, iters);
    return fmaf(vx, x, vy * y);
}

void orc_project_batch(const float *v, const float *theta, float *out,
                       long n, int iters) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; i++)
        out[i] = orc_project_n(v[2 * i], v[2 * i + 1], theta[i], iters);
}

/* lib/c/rac_cpu.c:322-328 (rac_sincos): rotate (RAC_K_INV, 0) by theta with
 * 16 iterations; (x, y) = (cos, sin). */
void orc_sincos(float theta, float *s, float *c) {
    float x = ORC_K_INV, y = 0.0f;
    orc_cordic_rotate(&x, &y, theta, ORC_ITERS);
    *c = x; *s = y;
}

/* lib/c/rac_cpu.c:576-598 (rac_rope_cache). */
void orc_rope_cache(float *cos_out, float *sin_out, int max_seq, int head_dim,
                    float base) {
    int half = head_dim / 2;
    #pragma omp parallel for schedule(static)
    for (int p = 0; p < max_seq; p++) {
        for (int i = 0; i < half; i++) {
            float exponent = (2.0f * (float)i) / (float)head_dim;
            float inv_freq = 1.0f / powf(base, exponent);
            float angle = (float)p * inv_freq;
            float s, c;
            orc_sincos(angle, &s, &c);
            cos_out[(long)p * half + i] = c;
            sin_out[(long)p * half + i] = s;
        }
    }
}

/* lib/c/rac_cpu.c:600-635 (rac_rope_apply), in place on [b, h, s, hd]. */
void orc_rope_apply(float *x, const float *cos_tab, const float *sin_tab,
                    int batch, int n_heads, int seq, int head_dim) {
    int half = head_dim / 2;
    long rows = (long)batch * n_heads * seq;
    #pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; r++) {
        int t = (int)(r % seq);
        float *row = x + r * head_dim;
        const float *cr = cos_tab + (long)t * half;
        const float *sr = sin_tab + (long)t * half;
        for (int i = 0; i < half; i++) {
            float a = row[2 * i], b = row[2 * i + 1];
            float c = cr[i], s = sr[i];
            row[2 * i]     = fmaf(a, c, -(b * s));
            row[2 * i + 1] = fmaf(a, s, b * c);
        }
    }
}

/* lib/c/rac_cpu.c:258-271 (rac_softmax) per row, :459-463 (batch). */
void orc_softmax_batch(const float *x, float *out, long rows, int n) {
    #pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; r++) {
        const float *xr = x + r * n;
        float *o = out + r * n;
        float m = xr[0];
        for (int i = 1; i < n; i++) if (xr[i] > m) m = xr[i];
        float sum = 0.0f;
        for (int i = 0; i < n; i++) { o[i] = expf(xr[i] - m); sum += o[i]; }
        float inv = 1.0f / sum;
        for (int i = 0; i < n; i++) o[i] *= inv;
    }
}

/* lib/c/rac_cpu.c:330-335 (rac_rsqrt). */
float orc_rsqrt(float x) { return x <= 0.0f ? 0.0f : 1.0f / sqrtf(x); }

/* lib/c/rac_cpu.c:548-574 (rac_rmsnorm); gamma may be NULL. */
void orc_rmsnorm(const float *x, float *y, const float *gamma, float eps,
                 long rows, int d) {
    #pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; r++) {
        const float *xr = x + r * d;
        float *yr = y + r * d;
        float ms = 0.0f;
        for (int i = 0; i < d; i++) ms = fmaf(xr[i], xr[i], ms);
        ms /= (float)d;
        float inv = orc_rsqrt(ms + eps);
        for (int i = 0; i < d; i++) {
            float g = gamma ? gamma[i] : 1.0f;
            yr[i] = xr[i] * inv * g;
        }
    }
}

/* lib/c/rac_cpu.c:507-546 (rac_layernorm); gamma/beta may be NULL. */
void orc_layernorm(const float *x, float *y, const float *gamma,
                   const float *beta, float eps, long rows, int d) {
    #pragma omp parallel for schedule(static)
    for (long r = 0; r < rows; r++) {
        const float *xr = x + r * d;
        float *yr = y + r * d;
        float mean = 0.0f;
        for (int i = 0; i < d; i++) mean += xr[i];
        mean /= (float)d;
        float var = 0.0f;
        for (int i = 0; i < d; i++) { float z = xr[i] - mean; var = fmaf(z, z, var); }
        var /= (float)d;
        float inv = orc_rsqrt(var + eps);
        for (int i = 0; i < d; i++) {
            float z = (xr[i] - mean) * inv;
            float g = gamma ? gamma[i] : 1.0f;
            float b = beta ? beta[i] : 0.0f;
            yr[i] = fmaf(g, z, b);
        }
    }
}

/* lib/c/rac_cpu.c:250-256 and :312-320: exp/tanh are libm on the CPU path
 * (the iteration count is ignored there). */
void orc_exp_batch(const float *x, float *y, long n) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; i++) y[i] = expf(x[i]);
}
void orc_tanh_batch(const float *x, float *y, long n) {
    #pragma omp parallel for schedule(static)
    for (long i = 0; i < n; i++) y[i] = tanhf(x[i]);
}

/* lib/c/rac_cpu.c:637-703 (rac_scaled_dot_attention): scores = (q.k)*scale
 * with fmaf over d, causal -inf above the diagonal, optional additive
 * [seq, seq] mask, row softmax (max, expf, sum, inv = sum > 0 ? 1/sum : 0),
 * out = sum_s fmaf(p, v, acc).  q, k, v, out: [batch, heads, seq, hd]. */
void orc_attention(const float *q, const float *k, const float *v, const float *mask,
                   int is_causal, float *out, int batch, int heads, int seq, int hd) {
    float scale = 1.0f / sqrtf((float)hd);
    #pragma omp parallel for collapse(2) schedule(dynamic)
    for (int b = 0; b < batch; b++) {
        for (int h = 0; h < heads; h++) {
            float *row = (float *)malloc((size_t)seq * sizeof(float));
            long base = ((long)(b * heads + h) * seq) * hd;
            const float *qb = q + base, *kb = k + base, *vb = v + base;
            float *ob = out + base;
            for (int t = 0; t < seq; t++) {
                for (int s2 = 0; s2 < seq; s2++) {
                    float acc = 0.0f;
                    for (int d = 0; d < hd; d++)
                        acc = fmaf(qb[(long)t * hd + d], kb[(long)s2 * hd + d], acc);
                    float sc = acc * scale;
                    if (is_causal && s2 > t) sc = -INFINITY;
                    if (mask) sc += mask[(long)t * seq + s2];
                    row[s2] = sc;
                }
                float m = row[0];
                for (int s2 = 1; s2 < seq; s2++) if (row[s2] > m) m = row[s2];
                float sum = 0.0f;
                for (int s2 = 0; s2 < seq; s2++) { row[s2] = expf(row[s2] - m); sum += row[s2]; }
                float inv = (sum > 0.0f) ? 1.0f / sum : 0.0f;
                for (int s2 = 0; s2 < seq; s2++) row[s2] *= inv;
                for (int d = 0; d < hd; d++) {
                    float acc = 0.0f;
                    for (int s2 = 0; s2 < seq; s2++) acc = fmaf(row[s2], vb[(long)s2 * hd + d], acc);
                    ob[(long)t * hd + d] = acc;
                }
            }
            free(row);
        }
    }
}

/* ── GEMM ──────────────────────────────────────────────────────────────────
 * rac_torch/rac_kernels.hip:139-185 (rac_cordic_rotate_n + rac_fma_cordic):
 * one MAC rotates (a, 0) by angle(b) in {0, pi}, runs `iters` micro-rotations,
 * multiplies the x component by 1/K(iters) and accumulates
 * fmaf(x * k_inv, |b|, acc).  The GEMM kernels of that file accumulate each
 * output sequentially over k (rac_kernels.hip:239-425), which this
 * restatement follows, so the GPU kernels match it bit for bit.
 *
 * layout: 0 = NN (A[M,K], B[K,N]), 1 = NT (B stored [N,K]),
 *         2 = TN (A stored [K,M]).
 * mode:   0 = FAST (sign-XOR FMA, rac_kernels.hip:56-64), 1 = CORDIC,
 *         2 = SHIFTADD (rac_kernels.hip:84-122, 217-218).
 */
static float orc_fma_cordic(float a, float b, float acc, int iters,
                            float k_inv) {
    uint32_t bi; memcpy(&bi, &b, 4);
    uint32_t mi = bi & 0x7FFFFFFFu;
    float mag_b; memcpy(&mag_b, &mi, 4);
    float theta = (bi & 0x80000000u) ? ORC_PI : 0.0f;
    float x = a, y = 0.0f;
    /* rac_kernels.hip:132-150: wrap (never triggers for 0 / pi) and fold. */
    orc_cordic_rotate(&x, &y, theta, iters);
    return fmaf(x * k_inv, mag_b, acc);
}

static float orc_fma_fast(float a, float b, float acc) {
    uint32_t ai, bi; memcpy(&ai, &a, 4); memcpy(&bi, &b, 4);
    uint32_t pi = ai ^ (bi & 0x80000000u), mi = bi & 0x7FFFFFFFu;
    float proj, mag; memcpy(&proj, &pi, 4); memcpy(&mag, &mi, 4);
    return fmaf(proj, mag, acc);
}

/* rac_torch/rac_kernels.hip:84-122 (rac_shiftadd_mul): a*b from the top
 * `iters` bits of b's 24-bit mantissa by integer shift-and-add, truncated
 * (no rounding) into an fp32 with sub/super-normal results flushed to 0.
 * Mode 2 of the GEMM accumulates acc + prod (rac_kernels.hip:217-218). */
float orc_shiftadd_mul(float a, float b, int iters) {
    if (a == 0.0f || b == 0.0f) return 0.0f;
    uint32_t ai, bi; memcpy(&ai, &a, 4); memcpy(&bi, &b, 4);
    uint32_t sign = (ai ^ bi) & 0x80000000u;
    int exp_a = (int)((ai >> 23) & 0xFFu) - 127;
    int exp_b = (int)((bi >> 23) & 0xFFu) - 127;
    uint32_t ma = 0x00800000u | (ai & 0x007FFFFFu);
    uint32_t mb = 0x00800000u | (bi & 0x007FFFFFu);
    uint64_t prod = 0;
    int lim = iters < 1 ? 1 : (iters > 24 ? 24 : iters);
    for (int i = 0; i < lim; i++) {
        uint32_t bit = (mb >> (23 - i)) & 1u;
        if (bit) prod += ((uint64_t)ma) << (23 - i);
    }
    if (prod == 0) return 0.0f;
    int top = 63 - __builtin_clzll(prod);
    int shift_r = top - 23;
    uint32_t mantissa;
    if (shift_r > 0) mantissa = (uint32_t)(prod >> shift_r) & 0x007FFFFFu;
    else if (shift_r < 0) mantissa = (uint32_t)(prod << -shift_r) & 0x007FFFFFu;
    else mantissa = (uint32_t)prod & 0x007FFFFFu;
    int rexp = exp_a + exp_b + (top - 46) + 127;
    if (rexp <= 0 || rexp >= 0xFF) return 0.0f;
    uint32_t bits = sign | ((uint32_t)(rexp & 0xFF) << 23) | mantissa;
    float r; memcpy(&r, &bits, 4);
    return r;
}

void orc_gemm(const float *A, const float *B, float *C, int M, int N, int K,
              int layout, int mode, int iters, long row0, long row1) {
    iters = orc_clamp_iters_gemm(iters);
    float k_inv = 1.0f / orc_k[iters];
    if (row1 <= 0 || row1 > M) row1 = M;
    #pragma omp parallel for schedule(dynamic, 1)
    for (long m = row0; m < row1; m++) {
        for (int n = 0; n < N; n++) {
            float acc = 0.0f;
            for (int k = 0; k < K; k++) {
                float a = (layout == 2) ? A[(long)k * M + m] : A[m * (long)K + k];
                float b = (layout == 1) ? B[(long)n * K + k] : B[(long)k * N + n];
                acc = mode == 1 ? orc_fma_cordic(a, b, acc, iters, k_inv)
                    : mode == 2 ? acc + orc_shiftadd_mul(a, b, iters)
                    : orc_fma_fast(a, b, acc);
            }
            C[(m - row0) * (long)N + n] = acc;
        }
    }
}

/* The CORDIC GEMM composed from lib/c's own primitive (no CORDIC GEMM exists
 * in lib/c): C[m,n] = sum_k rac_project_n((A[m,k], 0), B<0 ? pi : 0, n)*|B|
 * (lib/c/rac_cpu.c:282-288 with the encoding of rac_cuda.cu:594-611),
 * accumulated in double and rounded once.  NN layout; rows [row0, row1). */
void orc_gemm_composed(const float *A, const float *B, float *C, int M, int N,
                       int K, int iters, long row0, long row1) {
    if (row1 <= 0 || row1 > M) row1 = M;
    #pragma omp parallel for schedule(dynamic, 1)
    for (long m = row0; m < row1; m++) {
        for (int n = 0; n < N; n++) {
            double acc = 0.0;
            for (int k = 0; k < K; k++) {
                float b = B[(long)k * N + n];
                float th = (b < 0.0f) ? ORC_PI : 0.0f;
                acc += (double)orc_project_n(A[m * (long)K + k], 0.0f, th, iters)
                       * (double)fabsf(b);
            }
            C[(m - row0) * (long)N + n] = (float)acc;
        }
    }
}

/* Same composition, but calling a caller-supplied project_n (the reference
 * library's own rac_project_n, resolved from oracle/_ref by the caller).
 * This is the CPU CORDIC GEMM that the --impl reference bench leg times. */
typedef struct { float x, y; } orc_vec2;
typedef float (*orc_project_fn)(orc_vec2, float, int);
void orc_gemm_composed_with(orc_project_fn fn, const float *A, const float *B,
                            float *C, int M, int N, int K, int iters,
                            long row0, long row1) {
    if (row1 <= 0 || row1 > M) row1 = M;
    #pragma omp parallel for schedule(dynamic, 1)
    for (long m = row0; m < row1; m++) {
        for (int n = 0; n < N; n++) {
            float acc = 0.0f;
            for (int k = 0; k < K; k++) {
                float b = B[(long)k * N + n];
                orc_vec2 v = {A[m * (long)K + k], 0.0f};
                acc += fn(v, (b < 0.0f) ? ORC_PI : 0.0f, iters) * fabsf(b);
            }
            C[(m - row0) * (long)N + n] = acc;
        }
    }
}

int orc_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
