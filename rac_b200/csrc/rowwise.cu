// rowwise.cu -- softmax, RMSNorm and LayerNorm over rows of a row-major
// [rows, d] float32 matrix, for sm_100a.
//
// One CTA owns one row.  On the fast path (d % 4 == 0, 16-byte aligned,
// d <= 128 threads * 4 * MAXV) the whole row is loaded into registers with
// 128-bit streaming loads, reduced with warp shuffles plus one shared-memory
// exchange, and written once: every element crosses HBM exactly twice
// (read + write), the minimum.  Other shapes take a three-pass fallback that
// re-reads the row from global memory (L2-resident for d up to millions).
//
// Semantics: lib/c/rac_cpu.c:258-271 (softmax), :548-574 (rmsnorm),
// :507-546 (layernorm).  The per-element steps use the same rounding order;
// the row reductions are tree-ordered, so results differ from the
// sequential CPU sums by reduction rounding only (checked at 1e-4).
#include "rac_device.cuh"
#include "rac_internal.h"
#include "stream_ops.h"

namespace racb {

constexpr int kRowThreads = 128;
constexpr int kRowWarps = kRowThreads / 32;

enum RowOp : int { kRowSoftmax = 0, kRowRms = 1, kRowLayer = 2 };

template <bool IS_MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float w = __shfl_xor_sync(0xffffffffu, v, o);
        v = IS_MAX ? fmaxf(v, w) : __fadd_rn(v, w);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    __syncthreads();                       // red[] may still be read by a previous reduction
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float r = red[0];
#pragma unroll
    for (int w = 1; w < kRowWarps; ++w) r = IS_MAX ? fmaxf(r, red[w]) : __fadd_rn(r, red[w]);
    return r;
}

template <int OP, int V>
__global__ void __launch_bounds__(kRowThreads) k_row_vec(const float* __restrict__ x,
                                                         float* __restrict__ y,
                                                         const float* __restrict__ gamma,
                                                         const float* __restrict__ beta,
                                                         float eps, int d, long long rows) {
    __shared__ float red[kRowWarps];
    const int nq = d / 4;
    // One CTA per row (grid-stride if rows exceed the grid): the hardware
    // overlaps rows across CTAs.  gamma / beta are read through the read-only
    // path (L1 / L2 resident, 16 KB each at d = 4096); the loop issues the next
    // row's loads before the current row is reduced when a CTA owns several.
    const float fd = (float)d;
    float4 nxt[V];
    auto load_row = [&](long long r) {
        const float4* xr = reinterpret_cast<const float4*>(x + r * d);
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int q = threadIdx.x + j * kRowThreads;
            nxt[j] = (r < rows && q < nq) ? __ldcs(xr + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    load_row(blockIdx.x);
    for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    float4* yr = reinterpret_cast<float4*>(y + row * d);
    float4 v[V];
#pragma unroll
    for (int j = 0; j < V; ++j) v[j] = nxt[j];
    load_row(row + gridDim.x);           // in flight during this row's reductions
    if constexpr (OP == kRowSoftmax) {
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < V; ++j)
            if (threadIdx.x + j * kRowThreads < nq)
                m = fmaxf(fmaxf(m, fmaxf(v[j].x, v[j].y)), fmaxf(v[j].z, v[j].w));
        m = block_reduce<true>(m, red);
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j) {
            if (threadIdx.x + j * kRowThreads < nq) {
                v[j].x = expf(__fsub_rn(v[j].x, m)); v[j].y = expf(__fsub_rn(v[j].y, m));
                v[j].z = expf(__fsub_rn(v[j].z, m)); v[j].w = expf(__fsub_rn(v[j].w, m));
                sum = __fadd_rn(sum, __fadd_rn(__fadd_rn(v[j].x, v[j].y), __fadd_rn(v[j].z, v[j].w)));
            }
        }
        sum = block_reduce<false>(sum, red);
        const float inv = __fdiv_rn(1.0f, sum);
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int q = threadIdx.x + j * kRowThreads;
            if (q < nq)
                __stcs(yr + q, make_float4(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv),
                                           __fmul_rn(v[j].z, inv), __fmul_rn(v[j].w, inv)));
        }
    } else if constexpr (OP == kRowRms) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j) {
            ss = __fmaf_rn(v[j].x, v[j].x, ss); ss = __fmaf_rn(v[j].y, v[j].y, ss);
            ss = __fmaf_rn(v[j].z, v[j].z, ss); ss = __fmaf_rn(v[j].w, v[j].w, ss);
        }
        ss = block_reduce<false>(ss, red);
        const float ms = __fdiv_rn(ss, fd);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int q = threadIdx.x + j * kRowThreads;
            if (q < nq) {
                const float4 g = gamma ? __ldg(reinterpret_cast<const float4*>(gamma) + q)
                                       : make_float4(1.f, 1.f, 1.f, 1.f);
                __stcs(yr + q, make_float4(__fmul_rn(__fmul_rn(v[j].x, inv), g.x),
                                           __fmul_rn(__fmul_rn(v[j].y, inv), g.y),
                                           __fmul_rn(__fmul_rn(v[j].z, inv), g.z),
                                           __fmul_rn(__fmul_rn(v[j].w, inv), g.w)));
            }
        }
    } else {
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j)
            s = __fadd_rn(s, __fadd_rn(__fadd_rn(v[j].x, v[j].y), __fadd_rn(v[j].z, v[j].w)));
        s = block_reduce<false>(s, red);
        const float mean = __fdiv_rn(s, fd);
        float var = 0.0f;
#pragma unroll
        for (int j = 0; j < V; ++j) {
            if (threadIdx.x + j * kRowThreads < nq) {
                float z;
                z = __fsub_rn(v[j].x, mean); var = __fmaf_rn(z, z, var);
                z = __fsub_rn(v[j].y, mean); var = __fmaf_rn(z, z, var);
                z = __fsub_rn(v[j].z, mean); var = __fmaf_rn(z, z, var);
                z = __fsub_rn(v[j].w, mean); var = __fmaf_rn(z, z, var);
            }
        }
        var = block_reduce<false>(var, red);
        var = __fdiv_rn(var, fd);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
        for (int j = 0; j < V; ++j) {
            const int q = threadIdx.x + j * kRowThreads;
            if (q < nq) {
                const float4 g = gamma ? __ldg(reinterpret_cast<const float4*>(gamma) + q)
                                       : make_float4(1.f, 1.f, 1.f, 1.f);
                const float4 b = beta ? __ldg(reinterpret_cast<const float4*>(beta) + q)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                __stcs(yr + q, make_float4(
                    __fmaf_rn(g.x, __fmul_rn(__fsub_rn(v[j].x, mean), inv), b.x),
                    __fmaf_rn(g.y, __fmul_rn(__fsub_rn(v[j].y, mean), inv), b.y),
                    __fmaf_rn(g.z, __fmul_rn(__fsub_rn(v[j].z, mean), inv), b.z),
                    __fmaf_rn(g.w, __fmul_rn(__fsub_rn(v[j].w, mean), inv), b.w)));
            }
        }
    }
    }  // rows
}

// Any d, any alignment: reductions stream the row from global memory.
template <int OP>
__global__ void __launch_bounds__(kRowThreads) k_row_any(const float* __restrict__ x,
                                                         float* __restrict__ y,
                                                         const float* __restrict__ gamma,
                                                         const float* __restrict__ beta,
                                                         float eps, int d) {
    __shared__ float red[kRowWarps];
    const float* xr = x + (long long)blockIdx.x * d;
    float* yr = y + (long long)blockIdx.x * d;
    const float fd = (float)d;
    if constexpr (OP == kRowSoftmax) {
        float m = -INFINITY;
        for (int i = threadIdx.x; i < d; i += kRowThreads) m = fmaxf(m, xr[i]);
        m = block_reduce<true>(m, red);
        float sum = 0.0f;
        for (int i = threadIdx.x; i < d; i += kRowThreads) sum = __fadd_rn(sum, expf(__fsub_rn(xr[i], m)));
        sum = block_reduce<false>(sum, red);
        const float inv = __fdiv_rn(1.0f, sum);
        for (int i = threadIdx.x; i < d; i += kRowThreads)
            yr[i] = __fmul_rn(expf(__fsub_rn(xr[i], m)), inv);
    } else if constexpr (OP == kRowRms) {
        float ss = 0.0f;
        for (int i = threadIdx.x; i < d; i += kRowThreads) ss = __fmaf_rn(xr[i], xr[i], ss);
        ss = block_reduce<false>(ss, red);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, fd), eps)));
        for (int i = threadIdx.x; i < d; i += kRowThreads)
            yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), gamma ? gamma[i] : 1.0f);
    } else {
        float s = 0.0f;
        for (int i = threadIdx.x; i < d; i += kRowThreads) s = __fadd_rn(s, xr[i]);
        s = block_reduce<false>(s, red);
        const float mean = __fdiv_rn(s, fd);
        float var = 0.0f;
        for (int i = threadIdx.x; i < d; i += kRowThreads) {
            const float z = __fsub_rn(xr[i], mean);
            var = __fmaf_rn(z, z, var);
        }
        var = block_reduce<false>(var, red);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var, fd), eps)));
        for (int i = threadIdx.x; i < d; i += kRowThreads)
            yr[i] = __fmaf_rn(gamma ? gamma[i] : 1.0f, __fmul_rn(__fsub_rn(xr[i], mean), inv),
                              beta ? beta[i] : 0.0f);
    }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// One CTA per row.  Measured at [16384, 4096] against persistent CTAs that
// staged gamma / beta in shared memory once: RMSNorm 0.0891 ms vs 0.0959
// (persistent) / 0.0895 (8x oversubscribed), LayerNorm 0.0901 vs 0.0924;
// softmax was already one CTA per row.
template <int OP, int V>
static void launch_vec(const float* x, float* y, const float* g, const float* b, float eps,
                       int d, long long rows, cudaStream_t s) {
    const long long grid = rows > 0x7fffffffLL ? 0x7fffffffLL : rows;
    k_row_vec<OP, V><<<(unsigned)grid, kRowThreads, 0, s>>>(x, y, g, b, eps, d, rows);
}

template <int OP>
static int launch_rows(const float* x, float* y, const float* g, const float* b, float eps,
                       long long rows, int d, cudaStream_t s) {
    if (rows < 0 || d <= 0) return kErrInvalidDim;
    if (rows == 0) return kOk;
    if (!x || !y) return kErrNullPtr;
    if (rows > 0x7fffffffLL) return kErrInvalidDim;
    const bool vec = (d % 4 == 0) && al16(x) && al16(y) && (!g || al16(g)) && (!b || al16(b));
    const int nq = d / 4;
    if (vec && nq <= kRowThreads * 1) launch_vec<OP, 1>(x, y, g, b, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 2) launch_vec<OP, 2>(x, y, g, b, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 4) launch_vec<OP, 4>(x, y, g, b, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 8) launch_vec<OP, 8>(x, y, g, b, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 16) launch_vec<OP, 16>(x, y, g, b, eps, d, rows, s);
    else k_row_any<OP><<<dim3((unsigned)rows), kRowThreads, 0, s>>>(x, y, g, b, eps, d);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int softmax_rows(const float* x, float* y, long long rows, int d, cudaStream_t s) {
    return launch_rows<kRowSoftmax>(x, y, nullptr, nullptr, 0.0f, rows, d, s);
}
int rmsnorm_rows(const float* x, float* y, const float* gamma, float eps, long long rows, int d,
                 cudaStream_t s) {
    return launch_rows<kRowRms>(x, y, gamma, nullptr, eps, rows, d, s);
}
int layernorm_rows(const float* x, float* y, const float* gamma, const float* beta, float eps,
                   long long rows, int d, cudaStream_t s) {
    return launch_rows<kRowLayer>(x, y, gamma, beta, eps, rows, d, s);
}

}  // namespace racb
