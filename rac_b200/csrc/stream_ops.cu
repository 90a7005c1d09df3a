// stream_ops.cu -- elementwise RAC kernels for sm_100a.
//
// All of these are HBM-streaming: each element is read once and written once,
// with 128-bit loads/stores (two float2 vectors or four scalars per access)
// and a grid-stride loop over a grid sized to the SM count.  The arithmetic
// follows lib/c/rac_cpu.c rounding step by rounding step (see
// rac_device.cuh), so results are bit-identical to the reference library.
#include <atomic>

#include "rac_device.cuh"
#include "rac_internal.h"
#include "stream_ops.h"

namespace racb {

__device__ unsigned int g_err_word;   // per device: bit 0 = wrap-loop overrun

unsigned int* device_error_word(int device) {
    // Looked up once per device (that device current), then read lock-free.
    static std::atomic<unsigned int*> cache[64] = {};
    if (device < 0 || device >= 64) return nullptr;
    unsigned int* w = cache[device].load(std::memory_order_acquire);
    if (!w) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_err_word) != cudaSuccess) { cudaGetLastError(); return nullptr; }
        w = static_cast<unsigned int*>(p);
        cache[device].store(w, std::memory_order_release);
    }
    return w;
}

// Grid of a grid-stride kernel: per_sm CTAs of 256 threads per SM (at most
// 6-8 are resident at once).  8 suits the elementwise kernels (RoPE measured
// best there); the rotate kernels use 32: the later CTAs fill SMs whose
// earlier CTAs finished, and 2^26 vectors at n = 8 / 16 / 24 measured
// 0.217 / 0.227 / 0.304 ms against 0.249 / 0.239 / 0.310 ms with 8.
constexpr int kRotateCtasPerSm = 32;
static int grid_for(long long work_items, int threads, int per_sm = 8) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long blocks = (work_items + threads - 1) / threads;
    long long cap = (long long)sms * per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ── rotate / project / sincos ────────────────────────────────────────────

// (x, y) = rotation of (vx * k_inv, vy * k_inv) by th.
template <int ITERS>
__device__ __forceinline__ bool rotate_one(float& x, float& y, float vx, float vy, float k_inv,
                                           float th, int iters, unsigned sign_mask) {
    if constexpr (ITERS > 0) return cordic_rotate_scaled<ITERS>(x, y, vx, vy, k_inv, th, sign_mask);
    x = __fmul_rn(vx, k_inv);
    y = __fmul_rn(vy, k_inv);
    return cordic_rotate_rt(x, y, th, iters);
}

// out[i] = CORDIC rotation of (v[i] * k_inv) by theta[i]
// (lib/c/rac_cpu.c:136-139 with k_inv = RAC_K_INV, :275-280 with 1/K(n)).
template <int ITERS>
__global__ void __launch_bounds__(256) k_rotate(const float2* __restrict__ v,
                                                const float* __restrict__ th,
                                                float2* __restrict__ out, long long n,
                                                float k_inv, int iters, int vec,
                                                unsigned sign_mask) {
    bool ok = true;
    const long long stride = (long long)gridDim.x * blockDim.x;
    long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const long long nq = n / 4;
        // Software pipeline: the next quad's 48 bytes are requested before the
        // current quad's rotations run.
        float4 v01n = make_float4(0.f, 0.f, 0.f, 0.f), v23n = v01n, tn = v01n;
        if (i0 < nq) {
            v01n = __ldcs(reinterpret_cast<const float4*>(v) + 2 * i0);
            v23n = __ldcs(reinterpret_cast<const float4*>(v) + 2 * i0 + 1);
            tn = __ldcs(reinterpret_cast<const float4*>(th) + i0);
        }
        for (long long q = i0; q < nq; q += stride) {
            const float4 v01 = v01n, v23 = v23n, t = tn;
            if (q + stride < nq) {
                v01n = __ldcs(reinterpret_cast<const float4*>(v) + 2 * (q + stride));
                v23n = __ldcs(reinterpret_cast<const float4*>(v) + 2 * (q + stride) + 1);
                tn = __ldcs(reinterpret_cast<const float4*>(th) + q + stride);
            }
            float x0, y0, x1, y1, x2, y2, x3, y3;
            if constexpr (ITERS > 0) {                // two vectors per packed rotation
                ok &= cordic_rotate_scaled_x2<ITERS>(x0, y0, x1, y1, v01.x, v01.y, v01.z, v01.w,
                                                     k_inv, t.x, t.y, sign_mask);
                ok &= cordic_rotate_scaled_x2<ITERS>(x2, y2, x3, y3, v23.x, v23.y, v23.z, v23.w,
                                                     k_inv, t.z, t.w, sign_mask);
            } else {
                ok &= rotate_one<ITERS>(x0, y0, v01.x, v01.y, k_inv, t.x, iters, sign_mask);
                ok &= rotate_one<ITERS>(x1, y1, v01.z, v01.w, k_inv, t.y, iters, sign_mask);
                ok &= rotate_one<ITERS>(x2, y2, v23.x, v23.y, k_inv, t.z, iters, sign_mask);
                ok &= rotate_one<ITERS>(x3, y3, v23.z, v23.w, k_inv, t.w, iters, sign_mask);
            }
            __stcs(reinterpret_cast<float4*>(out) + 2 * q, make_float4(x0, y0, x1, y1));
            __stcs(reinterpret_cast<float4*>(out) + 2 * q + 1, make_float4(x2, y2, x3, y3));
        }
        i0 += nq * 4;   // the scalar tail below covers [4*nq, n)
        for (long long i = i0; i < n; i += stride) {
            const float2 vi = v[i];
            float x, y;
            ok &= rotate_one<ITERS>(x, y, vi.x, vi.y, k_inv, th[i], iters, sign_mask);
            out[i] = make_float2(x, y);
        }
    } else {
        for (long long i = i0; i < n; i += stride) {
            const float2 vi = v[i];
            float x, y;
            ok &= rotate_one<ITERS>(x, y, vi.x, vi.y, k_inv, th[i], iters, sign_mask);
            out[i] = make_float2(x, y);
        }
    }
    if (!ok) atomicOr(&g_err_word, 1u);
}

// out[i] = fmaf(v.x, c, v.y * s), (c, s) = rotation of (1/K(n), 0) by theta
// (lib/c/rac_cpu.c:282-288, rac_project_n).
template <int ITERS>
__global__ void __launch_bounds__(256) k_project(const float2* __restrict__ v,
                                                 const float* __restrict__ th,
                                                 float* __restrict__ out, long long n,
                                                 float k_inv, int iters, unsigned sign_mask) {
    bool ok = true;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float c, s;
        ok &= rotate_one<ITERS>(c, s, 1.0f, 0.0f, k_inv, th[i], iters, sign_mask);
        const float2 a = v[i];
        out[i] = __fmaf_rn(a.x, c, __fmul_rn(a.y, s));
    }
    if (!ok) atomicOr(&g_err_word, 1u);
}

// rac_sincos (lib/c/rac_cpu.c:322-328): rotate (RAC_K_INV, 0), 16 iterations.
__global__ void __launch_bounds__(256) k_sincos(const float* __restrict__ th,
                                                float* __restrict__ s_out,
                                                float* __restrict__ c_out, long long n) {
    bool ok = true;
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        float c = kKInv, s = 0.0f;
        ok &= cordic_rotate<kDefaultIters>(c, s, th[i]);
        s_out[i] = s;
        c_out[i] = c;
    }
    if (!ok) atomicOr(&g_err_word, 1u);
}

template <int ITERS>
static void launch_rotate_t(const float2* v, const float* th, float2* out, long long n,
                            float k_inv, int iters, cudaStream_t s) {
    const bool vec = al16(v) && al16(th) && al16(out);
    const int g = grid_for(vec ? (n + 3) / 4 : n, 256, kRotateCtasPerSm);
    k_rotate<ITERS><<<g, 256, 0, s>>>(v, th, out, n, k_inv, iters, vec ? 1 : 0, 0x80000000u);
}

int rotate_batch(const float2* v, const float* th, float2* out, long long n, int iters,
                 int literal_kinv, cudaStream_t s) {
    if (n < 0) return kErrInvalidDim;
    if (n == 0) return kOk;
    if (!v || !th || !out) return kErrNullPtr;
    float k_inv;
    if (literal_kinv) { iters = kDefaultIters; k_inv = kKInv; }
    else { iters = iters < 4 ? 4 : (iters > 24 ? 24 : iters); k_inv = k_inv_of(iters); }
    switch (iters) {
        case 8:  launch_rotate_t<8>(v, th, out, n, k_inv, iters, s); break;
        case 16: launch_rotate_t<16>(v, th, out, n, k_inv, iters, s); break;
        case 24: launch_rotate_t<24>(v, th, out, n, k_inv, iters, s); break;
        default: launch_rotate_t<0>(v, th, out, n, k_inv, iters, s); break;
    }
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int project_batch(const float2* v, const float* th, float* out, long long n, int iters,
                  cudaStream_t s) {
    if (n < 0) return kErrInvalidDim;
    if (n == 0) return kOk;
    if (!v || !th || !out) return kErrNullPtr;
    iters = iters < 4 ? 4 : (iters > 24 ? 24 : iters);
    const float k_inv = k_inv_of(iters);
    switch (iters) {
        case 8:  k_project<8><<<grid_for(n, 256, kRotateCtasPerSm), 256, 0, s>>>(v, th, out, n, k_inv, iters, 0x80000000u); break;
        case 16: k_project<16><<<grid_for(n, 256, kRotateCtasPerSm), 256, 0, s>>>(v, th, out, n, k_inv, iters, 0x80000000u); break;
        case 24: k_project<24><<<grid_for(n, 256, kRotateCtasPerSm), 256, 0, s>>>(v, th, out, n, k_inv, iters, 0x80000000u); break;
        default: k_project<0><<<grid_for(n, 256, kRotateCtasPerSm), 256, 0, s>>>(v, th, out, n, k_inv, iters, 0x80000000u); break;
    }
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int sincos_batch(const float* th, float* s_out, float* c_out, long long n, cudaStream_t s) {
    if (n < 0) return kErrInvalidDim;
    if (n == 0) return kOk;
    if (!th || !s_out || !c_out) return kErrNullPtr;
    k_sincos<<<grid_for(n, 256), 256, 0, s>>>(th, s_out, c_out, n);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// ── unary maps: exp, tanh, rsqrt, sigmoid ───────────────────────────────
// lib/c computes these with libm (rac_cpu.c:250-256, :312-320, :330-340).
// exp and tanh are evaluated in double and rounded once to float, which is
// the correctly rounded result in all but astronomically rare cases; rsqrt
// is IEEE sqrt followed by an IEEE divide, exactly as 1.0f/sqrtf(x).
__device__ __forceinline__ float unary_op(float x, int op) {
    switch (op) {
        case kUnaryExp: return (float)exp((double)x);
        case kUnaryTanh: return (float)tanh((double)x);
        case kUnaryRsqrt: return x <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(x));
        case kUnarySigmoid: {   // rac_cpu.c:337-340: 0.5f * (1.0f + tanhf(0.5f * x))
            const float t = (float)tanh((double)__fmul_rn(0.5f, x));
            return __fmul_rn(0.5f, __fadd_rn(1.0f, t));
        }
        default: return x;
    }
}

__global__ void __launch_bounds__(256) k_unary(const float* __restrict__ x, float* __restrict__ y,
                                               long long n, int op, int vec) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    long long i0 = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const long long nq = n / 4;
        for (long long q = i0; q < nq; q += stride) {
            float4 v = __ldcs(reinterpret_cast<const float4*>(x) + q);
            v.x = unary_op(v.x, op); v.y = unary_op(v.y, op);
            v.z = unary_op(v.z, op); v.w = unary_op(v.w, op);
            __stcs(reinterpret_cast<float4*>(y) + q, v);
        }
        i0 += nq * 4;
    }
    for (long long i = i0; i < n; i += stride) y[i] = unary_op(x[i], op);
}

int unary_batch(const float* x, float* y, long long n, int op, cudaStream_t s) {
    if (n < 0) return kErrInvalidDim;
    if (n == 0) return kOk;
    if (!x || !y) return kErrNullPtr;
    if (op < kUnaryExp || op > kUnarySigmoid) return kErrUnsupported;
    const bool vec = al16(x) && al16(y);
    k_unary<<<grid_for(vec ? (n + 3) / 4 : n, 256), 256, 0, s>>>(x, y, n, op, vec ? 1 : 0);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// ── RoPE ─────────────────────────────────────────────────────────────────

// rac_rope_cache (lib/c/rac_cpu.c:576-598):
//   inv_freq = 1 / powf(base, 2i/hd); angle = p * inv_freq; (c, s) = rac_sincos.
// powf is evaluated in double and rounded once (glibc's powf is correctly
// rounded on these arguments; the tests compare the tables bit for bit).
__global__ void __launch_bounds__(256) k_rope_cache(float* __restrict__ cos_out,
                                                    float* __restrict__ sin_out,
                                                    int max_seq, int head_dim, float base) {
    const int half = head_dim / 2;
    const long long total = (long long)max_seq * half;
    const long long stride = (long long)gridDim.x * blockDim.x;
    bool ok = true;
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += stride) {
        const int p = (int)(e / half), i = (int)(e % half);
        const float exponent = __fdiv_rn(__fmul_rn(2.0f, (float)i), (float)head_dim);
        const float pw = (float)pow((double)base, (double)exponent);
        const float inv_freq = __fdiv_rn(1.0f, pw);
        const float angle = __fmul_rn((float)p, inv_freq);
        float c = kKInv, s = 0.0f;
        ok &= cordic_rotate<kDefaultIters>(c, s, angle);
        cos_out[e] = c;
        sin_out[e] = s;
    }
    if (!ok) atomicOr(&g_err_word, 1u);
}

int rope_cache(float* cos_out, float* sin_out, int max_seq, int head_dim, float base,
               cudaStream_t s) {
    if (!cos_out || !sin_out) return kErrNullPtr;
    if (max_seq <= 0 || head_dim <= 0 || (head_dim & 1)) return kErrInvalidDim;
    const long long total = (long long)max_seq * (head_dim / 2);
    k_rope_cache<<<grid_for(total, 256), 256, 0, s>>>(cos_out, sin_out, max_seq, head_dim, base);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// Pair rotation of one (a, b) pair with table entries (c, s).
//   form 0 -- lib/c rac_rope_apply (rac_cpu.c:627-628):
//             (fmaf(a, c, -(b*s)), fmaf(a, s, b*c))
//   form 1 -- torch RACRoPE._apply_rotation (rac_torch/rac_torch.py:1177-1178):
//             (a*c - b*s, a*s + b*c), every product and sum rounded.
__device__ __forceinline__ float2 rope_pair(float a, float b, float c, float s, int form) {
    if (form == 0)
        return make_float2(__fmaf_rn(a, c, -__fmul_rn(b, s)), __fmaf_rn(a, s, __fmul_rn(b, c)));
    return make_float2(__fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s)),
                       __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c)));
}

// In place on rows of head_dim floats; row r has position
// pos[(r / seq) % pos_batch ...] -- here simply t = r % seq, or pos[t] when
// a position table is given.  Vector path: 4 floats (2 pairs) per access.
__global__ void __launch_bounds__(256) k_rope_apply(float* __restrict__ x,
                                                    const float* __restrict__ cos_tab,
                                                    const float* __restrict__ sin_tab,
                                                    const int* __restrict__ pos,
                                                    long long rows, int seq, int head_dim,
                                                    int form, int vec) {
    const int half = head_dim / 2;
    const long long stride = (long long)gridDim.x * blockDim.x;
    if (vec) {
        const int qpr = head_dim / 4;    // float4 per row
        const long long nq = rows * qpr;
        for (long long q = (long long)blockIdx.x * blockDim.x + threadIdx.x; q < nq; q += stride) {
            const long long r = q / qpr;
            const int j = (int)(q % qpr);           // pairs 2j, 2j+1
            int t = (int)(r % seq);
            if (pos) t = pos[t];
            float4 v = __ldcs(reinterpret_cast<const float4*>(x) + q);
            const float2 c = *reinterpret_cast<const float2*>(cos_tab + (long long)t * half + 2 * j);
            const float2 s = *reinterpret_cast<const float2*>(sin_tab + (long long)t * half + 2 * j);
            const float2 p0 = rope_pair(v.x, v.y, c.x, s.x, form);
            const float2 p1 = rope_pair(v.z, v.w, c.y, s.y, form);
            __stcs(reinterpret_cast<float4*>(x) + q, make_float4(p0.x, p0.y, p1.x, p1.y));
        }
    } else {
        const long long np = rows * half;
        for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < np; e += stride) {
            const long long r = e / half;
            const int i = (int)(e % half);
            int t = (int)(r % seq);
            if (pos) t = pos[t];
            float* row = x + r * head_dim;
            const float2 o = rope_pair(row[2 * i], row[2 * i + 1],
                                       cos_tab[(long long)t * half + i],
                                       sin_tab[(long long)t * half + i], form);
            row[2 * i] = o.x;
            row[2 * i + 1] = o.y;
        }
    }
}

int rope_apply(float* x, const float* cos_tab, const float* sin_tab, const int* pos,
               long long batch_heads, int seq, int head_dim, int form, cudaStream_t s) {
    if (!x || !cos_tab || !sin_tab) return kErrNullPtr;
    if (batch_heads <= 0 || seq <= 0 || head_dim <= 0 || (head_dim & 1)) return kErrInvalidDim;
    const long long rows = batch_heads * seq;
    const bool vec = (head_dim % 4 == 0) && al16(x) && ((reinterpret_cast<uintptr_t>(cos_tab) & 7u) == 0) &&
                     ((reinterpret_cast<uintptr_t>(sin_tab) & 7u) == 0);
    const long long work = vec ? rows * (head_dim / 4) : rows * (head_dim / 2);
    k_rope_apply<<<grid_for(work, 256), 256, 0, s>>>(x, cos_tab, sin_tab, pos, rows, seq,
                                                     head_dim, form, vec ? 1 : 0);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace racb
