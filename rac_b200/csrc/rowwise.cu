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
// :507-546 (layernorm).  The per-element steps use the same rounding order.
// Softmax and RMSNorm reduce their rows in tree order, so they differ from
// the sequential CPU sums by reduction rounding only (checked at 1e-4).
// LayerNorm cannot: y = gamma*z + beta cancels to ~0 wherever gamma*z ~ -beta,
// and there a one-ulp change of the row's mean or variance is a relative
// error far above 1e-4 (a tree-ordered LayerNorm measured 4.3e-4 from the
// reference at [16384, 4096]).  So LayerNorm reproduces lib/c's sequential
// mean and variance chains exactly (k_layernorm_seq below) and is
// bit-identical to it.
#include <cstdlib>

#include "rac_device.cuh"
#include "rac_internal.h"
#include "stream_ops.h"

namespace racb {

constexpr int kRowThreads = 128;
constexpr int kRowWarps = kRowThreads / 32;

enum RowOp : int { kRowSoftmax = 0, kRowRms = 1 };

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
    }
    }  // rows
}

// Any d, any alignment: reductions stream the row from global memory.
template <int OP>
__global__ void __launch_bounds__(kRowThreads) k_row_any(const float* __restrict__ x,
                                                         float* __restrict__ y,
                                                         const float* __restrict__ gamma,
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
    }
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// One CTA per row.  Measured at [16384, 4096] against persistent CTAs that
// staged gamma in shared memory once: RMSNorm 0.0891 ms vs 0.0959
// (persistent) / 0.0895 (8x oversubscribed); softmax was already one CTA
// per row.
template <int OP, int V>
static void launch_vec(const float* x, float* y, const float* g, float eps, int d,
                       long long rows, cudaStream_t s) {
    const long long grid = rows > 0x7fffffffLL ? 0x7fffffffLL : rows;
    k_row_vec<OP, V><<<(unsigned)grid, kRowThreads, 0, s>>>(x, y, g, eps, d, rows);
}

template <int OP>
static int launch_rows(const float* x, float* y, const float* g, float eps, long long rows, int d,
                       cudaStream_t s) {
    if (rows < 0 || d <= 0) return kErrInvalidDim;
    if (rows == 0) return kOk;
    if (!x || !y) return kErrNullPtr;
    if (rows > 0x7fffffffLL) return kErrInvalidDim;
    const bool vec = (d % 4 == 0) && al16(x) && al16(y) && (!g || al16(g));
    const int nq = d / 4;
    if (vec && nq <= kRowThreads * 1) launch_vec<OP, 1>(x, y, g, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 2) launch_vec<OP, 2>(x, y, g, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 4) launch_vec<OP, 4>(x, y, g, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 8) launch_vec<OP, 8>(x, y, g, eps, d, rows, s);
    else if (vec && nq <= kRowThreads * 16) launch_vec<OP, 16>(x, y, g, eps, d, rows, s);
    else k_row_any<OP><<<dim3((unsigned)rows), kRowThreads, 0, s>>>(x, y, g, eps, d);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// ── LayerNorm in lib/c's sequential order ─────────────────────────────────
// lib/c/rac_cpu.c:518-535 computes, per row, mean = (((x0 + x1) + x2) ...)/d
// and var = fmaf(z_{d-1}, z_{d-1}, ... fmaf(z0, z0, 0))/d with z = x - mean:
// two chains of d dependent roundings.  A chain cannot be split without
// changing its bits, so the kernel runs one chain per row, one row per lane,
// and gets its parallelism from many rows.
//
// A warp owns a group of 32 rows and streams it three times through a ring
// of kLnStages shared-memory chunks of 32 rows x 32 columns (cp.async,
// 16-byte pieces, coalesced in 128-byte row segments; row stride 36 floats,
// so each lane's 128-bit reads and writes of its own row are bank-conflict
// free): pass 0 runs the mean chains, pass 1 the variance chains, pass 2
// computes y = fmaf(gamma, (x - mean) * inv, beta) in the lane's row, writes
// it back into the chunk and stores the chunk with coalesced 128-bit stores.
// The loads form one continuous stream across passes and groups, kLnStages
// - 1 chunks ahead.  The kernel is persistent with few groups per SM in
// flight, so the second and third reads of a group come from L2: a group is
// 512 KB and is re-read within microseconds.  gamma and beta are staged in
// shared memory once per CTA when d <= kLnMaxD.
constexpr int kLnRows = 32;
constexpr int kLnChunk = 32;
constexpr int kLnLd = 36;
constexpr int kLnStages = 12;
constexpr int kLnMaxD = 4096;
constexpr int kLnCtasPerSm = 2;
constexpr int kLnRing = kLnStages * kLnRows * kLnLd;          // floats

__device__ __forceinline__ void ln_cp16(float* dst, const float* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 :: "r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))), "l"(src) : "memory");
}
__device__ __forceinline__ void ln_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void ln_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// rac_rsqrt of lib/c/rac_cpu.c:330-335.
__device__ __forceinline__ float ln_rsqrt(float v) {
    return v <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(v));
}

__global__ void __launch_bounds__(32) k_layernorm_seq(const float* __restrict__ x,
                                                      float* __restrict__ y,
                                                      const float* __restrict__ gamma,
                                                      const float* __restrict__ beta,
                                                      float eps, int d, long long rows) {
    extern __shared__ __align__(16) float smem[];
    float* ring = smem;
    const bool staged = d <= kLnMaxD;
    float* sg = smem + kLnRing;                 // gamma, beta (staged: d floats each)
    float* sb = sg + kLnMaxD;
    const int lane = threadIdx.x;
    const long long groups = (rows + kLnRows - 1) / kLnRows;
    const int nch = (d + kLnChunk - 1) / kLnChunk;
    const float fd = (float)d;
    if (staged) {
        for (int i = lane; i < d; i += 32) {
            sg[i] = gamma ? gamma[i] : 1.0f;
            sb[i] = beta ? beta[i] : 0.0f;
        }
    }
    // This CTA's chunk stream, group by group: pass 0, 1, 2 over chunks 0..nch-1.
    // Producer and consumer each walk it with counters (no divisions).
    const long long my_groups = groups > blockIdx.x ? (groups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    long long pg = blockIdx.x;                  // producer: group, pass, chunk, stage
    int ppass = 0, pc = 0, pst = 0;
    long long issued_groups = 0;
    auto issue = [&]() {
        if (issued_groups < my_groups) {
            const long long r0 = pg * kLnRows;
            const int nr = (int)(rows - r0 < kLnRows ? rows - r0 : kLnRows);
            float* st = ring + pst * (kLnRows * kLnLd);
#pragma unroll
            for (int i = 0; i < kLnRows * kLnChunk / 4 / 32; ++i) {
                const int idx = lane + 32 * i, rr = idx >> 3, q = idx & 7;
                const int col = pc * kLnChunk + 4 * q;
                if (rr < nr && col < d)
                    ln_cp16(st + rr * kLnLd + 4 * q, x + (r0 + rr) * (long long)d + col);
            }
            if (++pc == nch) {
                pc = 0;
                if (++ppass == 3) { ppass = 0; pg += gridDim.x; ++issued_groups; }
            }
        }
        if (++pst == kLnStages) pst = 0;
        ln_commit();                            // one group of copies per step, empty or not
    };
#pragma unroll 1
    for (int t = 0; t < kLnStages - 1; ++t) issue();
    __syncwarp();                               // gamma / beta staged
    float acc = 0.0f, mean = 0.0f, inv = 0.0f;
    long long cg = blockIdx.x;                  // consumer: group, pass, chunk, stage
    int pass = 0, c = 0, cst = 0;
#pragma unroll 1
    for (long long done = 0; done < my_groups;) {
        issue();
        ln_wait<kLnStages - 1>();               // this lane's pieces of the chunk landed
        __syncwarp();                           // ... and every other lane's
        if (c == 0) {
            if (pass == 0) acc = 0.0f;
            if (pass == 1) { mean = __fdiv_rn(acc, fd); acc = 0.0f; }   // mean /= (float)d
            if (pass == 2) inv = ln_rsqrt(__fadd_rn(__fdiv_rn(acc, fd), eps));
        }
        float* chunk = ring + cst * (kLnRows * kLnLd);
        float* rowp = chunk + lane * kLnLd;
        const int w = min(kLnChunk, d - c * kLnChunk);
        if (pass < 2) {
            if (w == kLnChunk) {
                float v[kLnChunk];
#pragma unroll
                for (int q = 0; q < kLnChunk / 4; ++q) {
                    const float4 f = *reinterpret_cast<const float4*>(rowp + 4 * q);
                    v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
                }
                if (pass == 0) {
#pragma unroll
                    for (int k = 0; k < kLnChunk; ++k) acc = __fadd_rn(acc, v[k]);
                } else {
#pragma unroll
                    for (int k = 0; k < kLnChunk; ++k) {
                        const float z = __fsub_rn(v[k], mean);
                        acc = __fmaf_rn(z, z, acc);
                    }
                }
            } else {
#pragma unroll 1
                for (int k = 0; k < w; ++k) {
                    const float vk = rowp[k];
                    if (pass == 0) acc = __fadd_rn(acc, vk);
                    else { const float z = __fsub_rn(vk, mean); acc = __fmaf_rn(z, z, acc); }
                }
            }
        } else {
            const int c0 = c * kLnChunk;
            // y for this lane's row, written back over x in the chunk
#pragma unroll 2
            for (int q = 0; q < w / 4; ++q) {
                const float4 f = *reinterpret_cast<const float4*>(rowp + 4 * q);
                float4 g4, b4;
                if (staged) {
                    g4 = *reinterpret_cast<const float4*>(sg + c0 + 4 * q);
                    b4 = *reinterpret_cast<const float4*>(sb + c0 + 4 * q);
                } else {
                    g4 = gamma ? __ldg(reinterpret_cast<const float4*>(gamma + c0) + q) : make_float4(1.f, 1.f, 1.f, 1.f);
                    b4 = beta ? __ldg(reinterpret_cast<const float4*>(beta + c0) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
                *reinterpret_cast<float4*>(rowp + 4 * q) =
                    make_float4(__fmaf_rn(g4.x, __fmul_rn(__fsub_rn(f.x, mean), inv), b4.x),
                                __fmaf_rn(g4.y, __fmul_rn(__fsub_rn(f.y, mean), inv), b4.y),
                                __fmaf_rn(g4.z, __fmul_rn(__fsub_rn(f.z, mean), inv), b4.z),
                                __fmaf_rn(g4.w, __fmul_rn(__fsub_rn(f.w, mean), inv), b4.w));
            }
            __syncwarp();                       // the chunk now holds y; store it coalesced
            const long long r0 = cg * kLnRows;
            const int nr = (int)(rows - r0 < kLnRows ? rows - r0 : kLnRows);
#pragma unroll
            for (int i = 0; i < kLnRows * kLnChunk / 4 / 32; ++i) {
                const int idx = lane + 32 * i, rr = idx >> 3, q = idx & 7;
                const int col = c0 + 4 * q;
                if (rr < nr && col < d)
                    __stcs(reinterpret_cast<float4*>(y + (r0 + rr) * (long long)d + col),
                           *reinterpret_cast<const float4*>(chunk + rr * kLnLd + 4 * q));
            }
        }
        __syncwarp();                           // the stage is re-filled next iteration
        if (++cst == kLnStages) cst = 0;
        if (++c == nch) {
            c = 0;
            if (++pass == 3) { pass = 0; cg += gridDim.x; ++done; }
        }
    }
    ln_wait<0>();
}

// Any d and alignment: one thread per row, the same chains straight from
// global memory (correct and exact, not fast).
__global__ void __launch_bounds__(128) k_layernorm_seq_any(const float* __restrict__ x,
                                                           float* __restrict__ y,
                                                           const float* __restrict__ gamma,
                                                           const float* __restrict__ beta,
                                                           float eps, int d, long long rows) {
    const long long r = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const float* xr = x + r * d;
    float* yr = y + r * d;
    float mean = 0.0f;
    for (int i = 0; i < d; ++i) mean = __fadd_rn(mean, xr[i]);
    mean = __fdiv_rn(mean, (float)d);
    float var = 0.0f;
    for (int i = 0; i < d; ++i) { const float z = __fsub_rn(xr[i], mean); var = __fmaf_rn(z, z, var); }
    const float inv = ln_rsqrt(__fadd_rn(__fdiv_rn(var, (float)d), eps));
    for (int i = 0; i < d; ++i)
        yr[i] = __fmaf_rn(gamma ? gamma[i] : 1.0f, __fmul_rn(__fsub_rn(xr[i], mean), inv),
                          beta ? beta[i] : 0.0f);
}

int softmax_rows(const float* x, float* y, long long rows, int d, cudaStream_t s) {
    return launch_rows<kRowSoftmax>(x, y, nullptr, 0.0f, rows, d, s);
}
int rmsnorm_rows(const float* x, float* y, const float* gamma, float eps, long long rows, int d,
                 cudaStream_t s) {
    return launch_rows<kRowRms>(x, y, gamma, eps, rows, d, s);
}
int layernorm_rows(const float* x, float* y, const float* gamma, const float* beta, float eps,
                   long long rows, int d, cudaStream_t s) {
    if (rows < 0 || d <= 0) return kErrInvalidDim;
    if (rows == 0) return kOk;
    if (!x || !y) return kErrNullPtr;
    const long long groups = (rows + kLnRows - 1) / kLnRows;
    const bool vec = (d % 4 == 0) && al16(x) && al16(y) && (!gamma || al16(gamma)) &&
                     (!beta || al16(beta));
    if (vec) {
        // Persistent: kLnCtasPerSm one-warp CTAs per SM, so that only that many
        // 512 KB row groups per SM are in flight and their re-reads hit L2.
        const int smem = (kLnRing + 2 * kLnMaxD) * (int)sizeof(float);
        static bool attr_set[64] = {};
        static int sms[64] = {};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) return kErrUnsupported;
        if (!attr_set[dev]) {
            if (cudaFuncSetAttribute(k_layernorm_seq, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     smem) != cudaSuccess) return kErrCuda;
            cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
            if (sms[dev] <= 0) sms[dev] = 148;
            attr_set[dev] = true;
        }
        int per_sm = kLnCtasPerSm;
        if (const char* e = getenv("RAC_LN_CTAS_PER_SM")) per_sm = atoi(e) > 0 ? atoi(e) : per_sm;
        long long grid = (long long)sms[dev] * per_sm;
        if (grid > groups) grid = groups;
        k_layernorm_seq<<<(unsigned)grid, 32, smem, s>>>(x, y, gamma, beta, eps, d, rows);
    } else {
        const long long blocks = (rows + 127) / 128;
        if (blocks > 0x7fffffffLL) return kErrInvalidDim;
        k_layernorm_seq_any<<<(unsigned)blocks, 128, 0, s>>>(x, y, gamma, beta, eps, d, rows);
    }
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace racb
