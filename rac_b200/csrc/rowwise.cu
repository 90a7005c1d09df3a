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
#include <atomic>

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
// and gets its parallelism from many rows.  Each row is therefore read three
// times (mean chain, variance chain, output) and written once.
//
// One persistent CTA per SM: kLnChains chain warps, each owning a group of 32
// rows (one per lane) at a time, and the remaining warps writing outputs.
//  * A chain warp streams its group twice through its own ring of kLnStages
//    shared-memory chunks of 32 rows x kLnCW columns.  Lane 0 fills a stage
//    with kLnCW / 32 TMA copies (cp.async.bulk.tensor.2d, a 32 x 32 box, the
//    128-byte swizzle, no multicast) that complete on the stage's mbarrier;
//    the swizzle puts lane r's 16-byte piece q of its row at slot q ^ (r & 7),
//    so the lanes' 128-bit reads of their own rows are bank-conflict free.
//    The reads run kLnNB float4 ahead of the chain (software pipelining),
//    so a chain step costs ~4.5 cycles, the dependent FADD / FFMA latency.
//    Pass 0 runs the mean chains, pass 1 the variance chains; the copies form
//    one continuous stream across passes and groups, kLnStages - 1 chunks
//    ahead.
//  * Meanwhile the output warps write y = fmaf(gamma, (x - mean) * inv, beta)
//    for the previous round's groups, row by row with coalesced 128-bit
//    accesses, kLnOut loads in flight per lane (gamma / beta staged in shared
//    memory).
//  * One __syncthreads per round hands the groups' mean / inv from the chain
//    warps to the output warps (double-buffered).
// Measured at [16384, 4096]: 0.188 ms, 1.01 GB of DRAM traffic (three reads
// and one write: a row's reads are too far apart for L2 to keep it), i.e.
// 5.4 TB/s, near that traffic's HBM floor of 0.155 ms; the tree-ordered
// one-read kernel this replaced ran in 0.090 ms but was 4.3e-4 (max-rel) from
// the reference.  Every mbarrier wait is bounded: a copy that never lands
// sets bit 2 of the device error word, and the warp stops issuing and drains
// (bounded) instead of hanging.
constexpr int kLnRows = 32;
constexpr int kLnThreads = 256;                                // chain warps first, then output
constexpr int kLnMaxGB = 4096;                                 // gamma / beta staged up to this d
constexpr int kLnOut = 16;                                     // output loads in flight per lane
constexpr int kLnNB = 8;                                       // float4 per chain batch
constexpr uint32_t kLnWaitLimit = 1u << 22;

__device__ __forceinline__ uint32_t ln_smem(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ bool ln_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(ln_smem(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// rac_rsqrt of lib/c/rac_cpu.c:330-335.
__device__ __forceinline__ float ln_rsqrt(float v) {
    return v <= 0.0f ? 0.0f : __fdiv_rn(1.0f, __fsqrt_rn(v));
}

// kLnCW: chunk width (floats, a multiple of 32); kLnStages: ring depth.
// tmx: x as a [rows, d] tensor map with a 32 x 32 box and the 128-byte swizzle.
template <int kLnCW, int kLnStages, int kLnChains>
__global__ void __launch_bounds__(kLnThreads) k_layernorm_seq(const __grid_constant__ CUtensorMap tmx,
                                                              const float* __restrict__ x,
                                                              float* __restrict__ y,
                                                              const float* __restrict__ gamma,
                                                              const float* __restrict__ beta,
                                                              float eps, int d, long long rows,
                                                              unsigned int* err) {
    static_assert(kLnCW % 32 == 0, "chunks are whole 32-column slabs");
    constexpr int kStage = kLnRows * kLnCW;                    // floats per stage
    extern __shared__ __align__(1024) float lnsm[];
    // the swizzled TMA destination wants 1024-byte alignment
    float* ring0 = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(lnsm) + 1023) & ~uintptr_t(1023));
    // gamma and beta staged after the rings when d <= kLnMaxGB (1 where absent)
    const bool staged = d <= kLnMaxGB;
    float* sg = ring0 + kLnChains * kLnStages * kStage;
    float* sb = sg + kLnMaxGB;
    __shared__ float s_mean[2][kLnChains * kLnRows], s_inv[2][kLnChains * kLnRows];
    __shared__ __align__(8) uint64_t fullb[kLnChains][kLnStages];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int cw = warp < kLnChains ? warp : 0;    // this chain warp's ring and barriers
    float* ring = ring0 + cw * kLnStages * kStage;
    uint64_t* full = fullb[cw];
    const long long groups = (rows + kLnRows - 1) / kLnRows;
    const long long my_groups = groups > blockIdx.x ? (groups - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int nch = (d + kLnCW - 1) / kLnCW;
    const float fd = (float)d;

    // chain warp: producer (bulk copies) and consumer (chains) positions
    long long pg = blockIdx.x + (long long)cw * gridDim.x, pgi = cw;
    int ppass = 0, pc = 0, pst = 0;
    int outstanding = 0;                        // chunks issued and not yet waited for
    bool bad = false;                           // a wait ran out: stop issuing, drain, report
    auto issue = [&]() {
        if (pgi < my_groups && !bad) {
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                             :: "r"(ln_smem(&full[pst])), "r"((uint32_t)(kStage * 4)) : "memory");
                float* dst = ring + pst * kStage;
#pragma unroll
                for (int sl = 0; sl < kLnCW / 32; ++sl)   // one 32 x 32 box per slab
                    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                                 " [%0], [%1, {%2, %3}], [%4];"
                                 :: "r"(ln_smem(dst + sl * 1024)), "l"(reinterpret_cast<uint64_t>(&tmx)),
                                    "r"(pc * kLnCW + 32 * sl), "r"((int)(pg * kLnRows)),
                                    "r"(ln_smem(&full[pst])) : "memory");
            }
            ++outstanding;
            if (++pc == nch) {
                pc = 0;
                if (++ppass == 2) { ppass = 0; pg += (long long)kLnChains * gridDim.x; pgi += kLnChains; }
            }
        }
        if (++pst == kLnStages) pst = 0;
    };
    if (warp < kLnChains) {
        if (lane == 0) {
            for (int st = 0; st < kLnStages; ++st)
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(ln_smem(&full[st])));
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncwarp();
        if (pgi < my_groups) {
#pragma unroll 1
            for (int t = 0; t < kLnStages - 1; ++t) issue();
        }
    }
    if (staged) {
        for (int i = threadIdx.x; i < d; i += kLnThreads) {
            sg[i] = gamma ? gamma[i] : 1.0f;
            sb[i] = beta ? beta[i] : 0.0f;
        }
    }
    __syncthreads();
    int cst = 0;
    uint32_t cpar = 0;                          // parity of the current use of the ring
#pragma unroll 1
    const long long rounds = (my_groups + kLnChains - 1) / kLnChains;
    for (long long k = 0; k <= rounds; ++k) {
        const int slot = (int)(k & 1);
        if (warp < kLnChains && k * kLnChains + warp < my_groups) {
            // ── chains of group k: pass 0 (mean), pass 1 (variance) ──
            float acc = 0.0f, mean = 0.0f;
#pragma unroll 1
            for (int pass = 0; pass < 2; ++pass) {
#pragma unroll 1
                for (int c = 0; c < nch; ++c) {
                    issue();
                    if (!bad) {
                        bool timed_out = false;
                        uint32_t polls = 0;
                        while (!ln_try_wait(&full[cst], cpar)) {
                            if (++polls >= kLnWaitLimit) { timed_out = true; break; }
                        }
                        if (__any_sync(0xffffffffu, timed_out)) {
                            // Report, then wait (bounded) for every copy still in
                            // flight, in issue order, so none lands after the CTA
                            // exits; from here on nothing is issued or awaited.
                            if (lane == 0 && err) atomicOr(err, 4u);
                            int s2 = cst;
                            uint32_t p2 = cpar;
                            for (int i = 0; i < outstanding; ++i) {
                                uint32_t n = 0;
                                while (!ln_try_wait(&full[s2], p2) && ++n < kLnWaitLimit) {}
                                if (++s2 == kLnStages) { s2 = 0; p2 ^= 1u; }
                            }
                            outstanding = 0;
                            bad = true;
                        } else {
                            --outstanding;
                        }
                    }
                    // lane's row: slab sl holds columns 32 sl .. 32 sl + 31 at
                    // rowp + sl * 1024; its 16-byte piece q sits at slot q ^ (lane & 7)
                    const float* rowp = ring + cst * kStage + lane * 32;
                    const int sw = lane & 7;
                    const int w = min(kLnCW, d - c * kLnCW);
                    if (w == kLnCW) {
                        // software-pipelined: the next kLnNB float4 of the row are
                        // read from shared memory while the chain runs on these
                        auto rd = [&](int u) {          // float4 u of the lane's row
                            return *reinterpret_cast<const float4*>(rowp + (u >> 3) * 1024 + (((u & 7) ^ sw) << 2));
                        };
                        float4 cur[kLnNB], nxt[kLnNB];
#pragma unroll
                        for (int u = 0; u < kLnNB; ++u) cur[u] = rd(u);
                        if (pass == 0) {
#pragma unroll
                            for (int bq = 0; bq < kLnCW / 4; bq += kLnNB) {
                                if (bq + kLnNB < kLnCW / 4) {
#pragma unroll
                                    for (int u = 0; u < kLnNB; ++u) nxt[u] = rd(bq + kLnNB + u);
                                }
#pragma unroll
                                for (int u = 0; u < kLnNB; ++u) {
                                    acc = __fadd_rn(acc, cur[u].x); acc = __fadd_rn(acc, cur[u].y);
                                    acc = __fadd_rn(acc, cur[u].z); acc = __fadd_rn(acc, cur[u].w);
                                }
#pragma unroll
                                for (int u = 0; u < kLnNB; ++u) cur[u] = nxt[u];
                            }
                        } else {
#pragma unroll
                            for (int bq = 0; bq < kLnCW / 4; bq += kLnNB) {
                                if (bq + kLnNB < kLnCW / 4) {
#pragma unroll
                                    for (int u = 0; u < kLnNB; ++u) nxt[u] = rd(bq + kLnNB + u);
                                }
#pragma unroll
                                for (int u = 0; u < kLnNB; ++u) {
                                    float z;
                                    z = __fsub_rn(cur[u].x, mean); acc = __fmaf_rn(z, z, acc);
                                    z = __fsub_rn(cur[u].y, mean); acc = __fmaf_rn(z, z, acc);
                                    z = __fsub_rn(cur[u].z, mean); acc = __fmaf_rn(z, z, acc);
                                    z = __fsub_rn(cur[u].w, mean); acc = __fmaf_rn(z, z, acc);
                                }
#pragma unroll
                                for (int u = 0; u < kLnNB; ++u) cur[u] = nxt[u];
                            }
                        }
                    } else {
#pragma unroll 1
                        for (int q = 0; q < w; ++q) {
                            const float vq = rowp[(q >> 5) * 1024 + ((((q >> 2) & 7) ^ sw) << 2) + (q & 3)];
                            if (pass == 0) acc = __fadd_rn(acc, vq);
                            else { const float z = __fsub_rn(vq, mean); acc = __fmaf_rn(z, z, acc); }
                        }
                    }
                    __syncwarp();               // every lane is done with the stage
                    if (++cst == kLnStages) { cst = 0; cpar ^= 1u; }
                }
                if (pass == 0) { mean = __fdiv_rn(acc, fd); acc = 0.0f; }   // mean /= (float)d
            }
            s_mean[slot][cw * kLnRows + lane] = mean;
            s_inv[slot][cw * kLnRows + lane] = ln_rsqrt(__fadd_rn(__fdiv_rn(acc, fd), eps));
        } else if (warp >= kLnChains && k >= 1) {
            // ── output of the previous round's groups ──
            const int ps = slot ^ 1;
            const int nq = d >> 2;
            const float4* g4 = reinterpret_cast<const float4*>(staged ? sg : gamma);
            const float4* b4 = reinterpret_cast<const float4*>(staged ? sb : beta);
            for (int ra = warp - kLnChains; ra < kLnChains * kLnRows; ra += kLnThreads / 32 - kLnChains) {
                const long long j = (k - 1) * kLnChains + ra / kLnRows;      // local group
                if (j >= my_groups) break;
                const int rr = ra % kLnRows;
                const long long r0 = ((long long)blockIdx.x + j * gridDim.x) * kLnRows;
                if (r0 + rr >= rows) continue;
                const float m = s_mean[ps][ra], inv = s_inv[ps][ra];
                const float4* xr = reinterpret_cast<const float4*>(x + (r0 + rr) * (long long)d);
                float4* yr = reinterpret_cast<float4*>(y + (r0 + rr) * (long long)d);
                // kLnOut loads of a lane in flight at once, then the stores
                for (int q0 = lane; q0 < nq; q0 += 32 * kLnOut) {
                    float4 v[kLnOut];
#pragma unroll
                    for (int u = 0; u < kLnOut; ++u) {
                        const int q = q0 + 32 * u;
                        v[u] = q < nq ? __ldcg(xr + q) : make_float4(0.f, 0.f, 0.f, 0.f);
                    }
#pragma unroll
                    for (int u = 0; u < kLnOut; ++u) {
                        const int q = q0 + 32 * u;
                        if (q < nq) {
                            const float4 g = g4 ? g4[q] : make_float4(1.f, 1.f, 1.f, 1.f);
                            const float4 b = b4 ? b4[q] : make_float4(0.f, 0.f, 0.f, 0.f);
                            __stcs(yr + q, make_float4(
                                __fmaf_rn(g.x, __fmul_rn(__fsub_rn(v[u].x, m), inv), b.x),
                                __fmaf_rn(g.y, __fmul_rn(__fsub_rn(v[u].y, m), inv), b.y),
                                __fmaf_rn(g.z, __fmul_rn(__fsub_rn(v[u].z, m), inv), b.z),
                                __fmaf_rn(g.w, __fmul_rn(__fsub_rn(v[u].w, m), inv), b.w)));
                        }
                    }
                }
            }
        }
        __syncthreads();                        // group k's stats -> output warps; slot reuse
    }
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
// One persistent CTA per SM (the grid never exceeds the number of groups).
template <int CW, int ST, int CH>
static int launch_ln(const float* x, float* y, const float* gamma, const float* beta, float eps,
                     int d, long long rows, int dev, cudaStream_t s) {
    const int smem = (CH * ST * kLnRows * CW + 2 * kLnMaxGB) * (int)sizeof(float) + 1024;
    CUtensorMap tmx;
    if (!encode_tensor_2d(&tmx, x, (uint64_t)d, (uint64_t)rows, d, 32, kLnRows, true)) return kErrUnsupported;
    static std::atomic<int> sms[64] = {};
    int n = sms[dev].load(std::memory_order_relaxed);
    if (!n) {
        if (cudaFuncSetAttribute(k_layernorm_seq<CW, ST, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 smem) != cudaSuccess) return kErrCuda;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
        sms[dev].store(n, std::memory_order_relaxed);
    }
    const long long groups = (rows + kLnRows - 1) / kLnRows;
    const long long grid = n < groups ? n : groups;
    k_layernorm_seq<CW, ST, CH><<<(unsigned)grid, kLnThreads, smem, s>>>(tmx, x, y, gamma, beta, eps, d,
                                                                        rows, device_error_word(dev));
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int layernorm_rows(const float* x, float* y, const float* gamma, const float* beta, float eps,
                   long long rows, int d, cudaStream_t s) {
    if (rows < 0 || d <= 0) return kErrInvalidDim;
    if (rows == 0) return kOk;
    if (!x || !y) return kErrNullPtr;
    const bool vec = (d % 4 == 0) && al16(x) && al16(y) && (!gamma || al16(gamma)) &&
                     (!beta || al16(beta));
    if (vec) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 0 || dev >= 64) return kErrUnsupported;
        // 2 chain warps, 128-column chunks, 4 stages each (measured against one chain
        // warp with 128 x 6 / 256 x 4 rings and two with 128 x 6: 0.189-0.223 ms)
        const int st = launch_ln<128, 4, 2>(x, y, gamma, beta, eps, d, rows, dev, s);
        if (st != kErrUnsupported) return st;
    }
    const long long blocks = (rows + 127) / 128;
    if (blocks > 0x7fffffffLL) return kErrInvalidDim;
    k_layernorm_seq_any<<<(unsigned)blocks, 128, 0, s>>>(x, y, gamma, beta, eps, d, rows);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace racb
