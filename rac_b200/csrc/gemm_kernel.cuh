// gemm_kernel.cuh -- the rotation-accumulate GEMM for sm_100a.
//
// C[M,N] = alpha * sum_k MAC(A[m,k], B[k,n]) (+ beta*Cin) (+ bias) -> act,
// where MAC is one of the reference's per-element products
// (rac_torch/rac_kernels.hip:203-219):
//   FAST   -- sign-XOR FMA (rac_kernels.hip:56-64).  (a ^ sign b) * |b| is
//             bit-identical to a * b, so it is issued as one FFMA.
//   CORDIC -- rac_fma_cordic (rac_kernels.hip:176-185): (a, 0) rotated by
//             angle(b) in {0, pi} through `iters` micro-rotations, x scaled
//             by 1/K(iters), accumulated as fmaf(x * k_inv, |b|, acc).
//
// The CORDIC MAC costs 2*iters FP32/INT instructions (1 LOP3 for the fold,
// 2*iters-3 FFMA for iterations 1..iters-1 -- iteration 0 is an exact copy --
// 1 FMUL, 1 FFMA), so the kernel is bound by the SM's FP32 pipe, not by
// memory: a 64x128 tile with K=4096 moves 3 MB from L2 for ~5e9 FP32
// operations.  The design therefore spends its effort on keeping that pipe
// fed: a register tile per thread gives 32-64 independent rotation chains for
// the scheduler to interleave, the fixed-n kernels run the micro-rotations of
// two rows as one FFMA2 (half the issue slots, so issue is no longer the
// limit), operands are staged through shared memory by TMA (or a register
// double buffer) so loads never sit on the issue path, and each output
// accumulates sequentially over k (the reference kernels' order), which keeps
// the result bit-identical to the CPU restatement.
// No tensor cores: the defining arithmetic is the micro-rotation, not a MAC.
#pragma once
#include "rac_device.cuh"
#include "rac_internal.h"

namespace racb {

__device__ __forceinline__ float apply_act(float x, int act) {
    // rac_torch/rac_torch.cu:668-676 (_apply_act).
    switch (act) {
        case kActRelu: return x > 0.0f ? x : 0.0f;
        case kActGelu: return x * 0.5f * (1.0f + erff(x * 0.7071067811865f));
        case kActSilu: return __fdiv_rn(x, 1.0f + expf(-x));
        default: return x;
    }
}

// Global -> register -> shared staging of one operand tile.
//   ROWS x COLS tile of a row-major matrix (COLS contiguous, leading dim ld),
//   stored into smem as S[k][mn] with k along COLS (TRANS) or along ROWS.
template <int ROWS, int COLS, int NT, bool VEC>
struct TileLoader {
    static constexpr int ELEMS = ROWS * COLS;
    static constexpr int PER = VEC ? 4 : 1;
    static constexpr int LOADS = (ELEMS + PER * NT - 1) / (PER * NT);
    static constexpr bool PARTIAL = (ELEMS % (PER * NT)) != 0;
    static_assert(!PARTIAL || LOADS == 1, "partial tiles only when a tile needs one pass");
    float r[LOADS * PER];

    __device__ __forceinline__ void load(const float* __restrict__ src, long long ld,
                                         int row0, int col0, int rows_lim, int cols_lim,
                                         int tid) {
#pragma unroll
        for (int l = 0; l < LOADS; ++l) {
            const int idx = (tid + l * NT) * PER;
            if (PARTIAL && idx >= ELEMS) break;
            const int rr = idx / COLS, cc = idx % COLS;
            const int gr = row0 + rr, gc = col0 + cc;
            if constexpr (VEC) {
                float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
                // cols_lim is a multiple of 4 on the VEC path, so a vector is
                // either fully inside or fully outside.
                if (gr < rows_lim && gc < cols_lim)
                    v = __ldg(reinterpret_cast<const float4*>(src + (long long)gr * ld + gc));
                r[l * 4 + 0] = v.x; r[l * 4 + 1] = v.y;
                r[l * 4 + 2] = v.z; r[l * 4 + 3] = v.w;
            } else {
                r[l] = (gr < rows_lim && gc < cols_lim) ? __ldg(src + (long long)gr * ld + gc) : 0.0f;
            }
        }
    }

    // K_ALONG_COLS: the tile's columns are k (store transposed: S[c][r]);
    // otherwise the tile's rows are k (S[r][c]).  S has row length SLD.
    template <bool K_ALONG_COLS, int SLD>
    __device__ __forceinline__ void store(float* S, int tid) const {
#pragma unroll
        for (int l = 0; l < LOADS; ++l) {
            const int idx = (tid + l * NT) * PER;
            if (PARTIAL && idx >= ELEMS) break;
            const int rr = idx / COLS, cc = idx % COLS;
            if constexpr (K_ALONG_COLS) {
#pragma unroll
                for (int q = 0; q < PER; ++q) S[(cc + q) * SLD + rr] = r[l * PER + q];
            } else {
                if constexpr (VEC) {
                    *reinterpret_cast<float4*>(&S[rr * SLD + cc]) =
                        make_float4(r[l * 4 + 0], r[l * 4 + 1], r[l * 4 + 2], r[l * 4 + 3]);
                } else {
                    S[rr * SLD + cc] = r[l];
                }
            }
        }
    }
};

// ── TMA staging (cp.async.bulk.tensor, no multicast) ──────────────────────
// Tensor maps are built on the host (gemm_dispatch.cu) and passed inside the
// __grid_constant__ parameters.  One elected thread issues the copies of a
// stage; every thread waits on that stage's mbarrier with a bounded loop.
__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(ptr));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
                    "r"(smem_u32(bar)) : "memory");
}
// Default upper bound on the polls of one stage barrier: a copy that never
// lands sets bit 1 of the device error word instead of hanging the kernel.
constexpr uint32_t kTmaWaitLimit = 1u << 22;

// Writes a thread's TM x TN register tile: raw partial sums to the split-K
// workspace, or the epilogue C = act(alpha*acc + beta*Cin + bias) (the
// SwiGLU pairing included).  acc(i, j) reads the thread's accumulator,
// row_of / col_of map tile indices to the CTA tile.
template <int TM, int TN, class AccF, class RowF, class ColF>
__device__ __forceinline__ void store_tile(const GemmParams& p, int m0, int n0, AccF acc,
                                           RowF row_of, ColF col_of) {
    if (p.ws) {   // split-K partial: raw sums, the reduction applies the epilogue
        float* w = p.ws + (long long)blockIdx.z * p.M * p.N;
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int gm = m0 + row_of(i);
            if (gm >= p.M) continue;
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                const int gn = n0 + col_of(j);
                if (gn < p.N) w[(long long)gm * p.N + gn] = acc(i, j);
            }
        }
        return;
    }
    // Epilogue (rac_kernels.hip:790-797 for alpha/beta; rac_torch.cu:769-776
    // for bias + activation).
    if (p.act == kActSwiGLU) {
        // Columns (2c, 2c+1) hold gate and up of output c; a thread's columns
        // come in groups of 4 consecutive ones starting at a multiple of 4, so
        // each pair is in one thread.  silu(gate) * up, each factor rounded as
        // the separate GEMM epilogue and the elementwise product would round it.
#pragma unroll
        for (int i = 0; i < TM; ++i) {
            const int gm = m0 + row_of(i);
            if (gm >= p.M) continue;
#pragma unroll
            for (int j = 0; j < TN; j += 2) {
                const int gn = n0 + col_of(j);
                if (gn >= p.N) continue;
                float g = __fmul_rn(p.alpha, acc(i, j)), u = __fmul_rn(p.alpha, acc(i, j + 1));
                if (p.bias) { g = __fadd_rn(g, p.bias[gn]); u = __fadd_rn(u, p.bias[gn + 1]); }
                p.C[(long long)gm * p.ldc + (gn >> 1)] = __fmul_rn(apply_act(g, kActSilu), u);
            }
        }
        return;
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int gm = m0 + row_of(i);
        if (gm >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int gn = n0 + col_of(j);
            if (gn >= p.N) continue;
            float v;
            if (p.beta != 0.0f)
                v = __fmaf_rn(p.alpha, acc(i, j), __fmul_rn(p.beta, p.Cin[(long long)gm * p.ldcin + gn]));
            else
                v = __fmul_rn(p.alpha, acc(i, j));
            if (p.bias) v = __fadd_rn(v, p.bias[gn]);
            if (p.act) v = apply_act(v, p.act);
            p.C[(long long)gm * p.ldc + gn] = v;
        }
    }
}

template <int MODE, int ITERS, int LAYOUT, int BM, int BN, int BK, int TM, int TN, bool VEC,
          int MINB = 1, bool TMA = false>
__global__ void __launch_bounds__((BM / TM) * (BN / TN), MINB)
k_gemm(const __grid_constant__ GemmParams p) {
    constexpr int TX = BN / TN, TY = BM / TM, NT = TX * TY;
    constexpr int STAGES = TMA ? 4 : 2;
    // A: NN/NT store A[M,K] (k contiguous); TN stores A[K,M].
    // B: NN/TN store B[K,N] (n contiguous); NT stores B[N,K].
    constexpr bool A_KCOLS = (LAYOUT != kTN);
    constexpr bool B_KCOLS = (LAYOUT == kNT);
    // Shared-memory layout of a stage.  The register-staged path transposes
    // into k-major rows; TMA copies the box as it lies in global memory, so
    // an operand whose global rows run along k lands m-/n-major.
    constexpr bool A_KMAJOR = TMA ? !A_KCOLS : true;
    constexpr bool B_KMAJOR = TMA ? !B_KCOLS : true;
    __shared__ __align__(128) float As[STAGES][BK * BM];
    __shared__ __align__(128) float Bs[STAGES][BK * BN];
    __shared__ __align__(8) uint64_t full_bar[TMA ? STAGES : 1];

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    // Ownership: a thread's TM rows (TN columns) are TM/4 (TN/4) groups of 4
    // consecutive rows (columns) spaced BM/(TM/4) (BN/(TN/4)) apart, so the
    // float4 shared-memory reads of a warp are contiguous (bank-conflict
    // free).  Which thread owns an output does not change its arithmetic.
    auto row_of = [&](int i) { return (i >> 2) * (BM / (TM / 4)) + ty * 4 + (i & 3); };
    auto col_of = [&](int j) { return (j >> 2) * (BN / (TN / 4)) + tx * 4 + (j & 3); };
    // K range of this CTA: all of K, or one split-K chunk (kchunk % BK == 0).
    const int kbeg = p.ws ? blockIdx.z * p.kchunk : 0;
    const int kend = p.ws ? min(p.K, kbeg + p.kchunk) : p.K;
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;   // m tiles on x (2^31 limit)

    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

    const float k_inv = p.k_inv;
    const int ktiles = (kend - kbeg + BK - 1) / BK;

    // One k-step of the register tile from stage buffers Asb / Bsb.
    auto mac_step = [&](const float* __restrict__ Asb, const float* __restrict__ Bsb, int kk) {
        float a[TM], b[TN];
        if constexpr (A_KMAJOR) {
#pragma unroll
            for (int i = 0; i < TM; i += 4) {
                const float4 v = *reinterpret_cast<const float4*>(&Asb[kk * BM + row_of(i)]);
                a[i] = v.x; a[i + 1] = v.y; a[i + 2] = v.z; a[i + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = Asb[row_of(i) * BK + kk];
        }
        if constexpr (B_KMAJOR) {
#pragma unroll
            for (int j = 0; j < TN; j += 4) {
                const float4 v = *reinterpret_cast<const float4*>(&Bsb[kk * BN + col_of(j)]);
                b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
            }
        } else {
#pragma unroll
            for (int j = 0; j < TN; ++j) b[j] = Bsb[col_of(j) * BK + kk];
        }
        if constexpr (MODE == kFast) {
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j)
                    acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        } else if constexpr (MODE == kShiftAdd) {
            // rac_fma_iters SHIFTADD (rac_kernels.hip:217-218): acc + prod.
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j)
                    acc[i][j] = __fadd_rn(acc[i][j], shiftadd_mul(a[i], b[j], p.iters));
        } else {
            uint32_t sgn[TN];
            float mag[TN];
#pragma unroll
            for (int j = 0; j < TN; ++j) {
                sgn[j] = __float_as_uint(b[j]) & 0x80000000u;
                mag[j] = __uint_as_float(__float_as_uint(b[j]) & 0x7FFFFFFFu);
            }
            if constexpr (ITERS > 0 && (TM % 2) == 0) {
                // two rows' micro-rotations per FFMA2
                const float2 ki2 = make_float2(k_inv, k_inv);
#pragma unroll
                for (int j = 0; j < TN; ++j) {
#pragma unroll
                    for (int i = 0; i < TM; i += 2) {
                        const float2 sa = make_float2(__uint_as_float(__float_as_uint(a[i]) ^ sgn[j]),
                                                      __uint_as_float(__float_as_uint(a[i + 1]) ^ sgn[j]));
                        const float2 xs = __fmul2_rn(gemm_cordic_x2<ITERS>(sa), ki2);
                        acc[i][j] = __fmaf_rn(xs.x, mag[j], acc[i][j]);
                        acc[i + 1][j] = __fmaf_rn(xs.y, mag[j], acc[i + 1][j]);
                    }
                }
            } else {
#pragma unroll
            for (int j = 0; j < TN; ++j) {
#pragma unroll
                for (int i = 0; i < TM; ++i) {
                    const float sa = __uint_as_float(__float_as_uint(a[i]) ^ sgn[j]);
                    float x;
                    if constexpr (ITERS > 0) x = gemm_cordic_x<ITERS>(sa);
                    else                     x = gemm_cordic_x_rt(sa, p.iters, p.coef);
                    acc[i][j] = __fmaf_rn(__fmul_rn(x, k_inv), mag[j], acc[i][j]);
                }
            }
            }
        }
    };

    if constexpr (TMA) {
        constexpr uint32_t kStageBytes = sizeof(float) * (BM + BN) * BK;
        auto issue = [&](int stage, int k0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(&full_bar[stage], kStageBytes + p.tma_extra_tx);
            if constexpr (A_KCOLS) tma_load_2d(As[stage], &p.tmA, k0, m0, &full_bar[stage]);
            else                   tma_load_2d(As[stage], &p.tmA, m0, k0, &full_bar[stage]);
            if constexpr (B_KCOLS) tma_load_2d(Bs[stage], &p.tmB, k0, n0, &full_bar[stage]);
            else                   tma_load_2d(Bs[stage], &p.tmB, n0, k0, &full_bar[stage]);
        };
        if (tid == 0) {
#pragma unroll
            for (int st = 0; st < STAGES; ++st) mbar_init(&full_bar[st], 1);
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
        __syncthreads();
        if (tid == 0)
            for (int st = 0; st < STAGES && st < ktiles; ++st) issue(st, kbeg + st * BK);
        bool timed_out = false;
        for (int kt = 0; kt < ktiles; ++kt) {
            const int st = kt % STAGES;
            const uint32_t parity = (kt / STAGES) & 1u;
            if (!timed_out) {
                uint32_t polls = 0;
                while (!mbar_try_wait(&full_bar[st], parity)) {
                    if (++polls >= p.tma_wait_limit) { timed_out = true; break; }
                }
            }
#pragma unroll 1
            for (int kk = 0; kk < BK; ++kk) mac_step(As[st], Bs[st], kk);
            __syncthreads();                       // every thread is done with stage st
            // After a timeout the stage's phase never completed; re-arming it
            // would arrive on a barrier with no pending arrivals, so stop.
            if (tid == 0 && !timed_out && kt + STAGES < ktiles) issue(st, kbeg + (kt + STAGES) * BK);
        }
        if (timed_out && p.err) atomicOr(p.err, 2u);
    } else {
        TileLoader<A_KCOLS ? BM : BK, A_KCOLS ? BK : BM, NT, VEC> la;
        TileLoader<B_KCOLS ? BN : BK, B_KCOLS ? BK : BN, NT, VEC> lb;
        auto load_tiles = [&](int k0) {
            if constexpr (A_KCOLS) la.load(p.A, p.lda, m0, k0, p.M, kend, tid);
            else                   la.load(p.A, p.lda, k0, m0, kend, p.M, tid);
            if constexpr (B_KCOLS) lb.load(p.B, p.ldb, n0, k0, p.N, kend, tid);
            else                   lb.load(p.B, p.ldb, k0, n0, kend, p.N, tid);
        };
        auto store_tiles = [&](int buf) {
            la.template store<A_KCOLS, BM>(As[buf], tid);
            lb.template store<B_KCOLS, BN>(Bs[buf], tid);
        };
        load_tiles(kbeg);
        store_tiles(0);
        __syncthreads();
        for (int kt = 0; kt < ktiles; ++kt) {
            const int buf = kt & 1;
            if (kt + 1 < ktiles) load_tiles(kbeg + (kt + 1) * BK);   // in flight during compute
#pragma unroll 1
            for (int kk = 0; kk < BK; ++kk) mac_step(As[buf], Bs[buf], kk);
            if (kt + 1 < ktiles) store_tiles(buf ^ 1);
            __syncthreads();
        }
    }

    store_tile<TM, TN>(p, m0, n0, [&](int i, int j) { return acc[i][j]; }, row_of, col_of);
}

// Tile variants.  1: 64x128 CTA tile, 8x8 per thread (the general case);
// 3: 16x128, 4x4 per thread (M <= 32, e.g. decode-shaped rows).
template <int V> struct TileCfg;
// 2: 64x64, 8x4 per thread, for mid-size problems whose 64x128 tiles would
// leave resident slots empty (2048^3: 512 tiles for 592 slots).
// MINB: resident CTAs per SM the register budget is sized for.
template <> struct TileCfg<1> { static constexpr int BM = 64, BN = 128, BK = 8, TM = 8, TN = 8, MINB = 4; };
template <> struct TileCfg<2> { static constexpr int BM = 64, BN = 64, BK = 8, TM = 8, TN = 4, MINB = 6; };
template <> struct TileCfg<3> { static constexpr int BM = 16, BN = 128, BK = 8, TM = 4, TN = 4, MINB = 4; };
// 4: 32x64, 4x4 per thread: finer tiles for narrow shards (4096x512 per GPU).
template <> struct TileCfg<4> { static constexpr int BM = 32, BN = 64, BK = 8, TM = 4, TN = 4, MINB = 8; };

template <int MODE, int ITERS, int LAYOUT, int V, bool VEC, bool TMA = false>
int launch_inst(const GemmParams& p_in, cudaStream_t s) {
    using T = TileCfg<V>;
    constexpr int NT = (T::BM / T::TM) * (T::BN / T::TN);
    dim3 grid((p_in.M + T::BM - 1) / T::BM, (p_in.N + T::BN - 1) / T::BN, p_in.ws ? p_in.splits : 1);
    if (grid.y > 65535) return kErrInvalidDim;
    if constexpr (TMA) {
        GemmParams p = p_in;
        if (!make_tensor_maps(p, LAYOUT, T::BM, T::BN, T::BK)) return kErrUnsupported;
        k_gemm<MODE, ITERS, LAYOUT, T::BM, T::BN, T::BK, T::TM, T::TN, VEC, T::MINB, true><<<grid, NT, 0, s>>>(p);
    } else {
        k_gemm<MODE, ITERS, LAYOUT, T::BM, T::BN, T::BK, T::TM, T::TN, VEC, T::MINB><<<grid, NT, 0, s>>>(p_in);
    }
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// Explicit instantiations live in gemm_inst_*.cu so that the heavy unrolled
// kernels compile in parallel translation units.
#define RACB_GEMM_INST(MODE, ITERS, LAYOUT, V, VEC) \
    template int launch_inst<MODE, ITERS, LAYOUT, V, VEC>(const GemmParams&, cudaStream_t);
#define RACB_GEMM_EXTERN(MODE, ITERS, LAYOUT, V, VEC) \
    extern template int launch_inst<MODE, ITERS, LAYOUT, V, VEC>(const GemmParams&, cudaStream_t);
#define RACB_GEMM_INST_TMA(MODE, ITERS, LAYOUT, V) \
    template int launch_inst<MODE, ITERS, LAYOUT, V, true, true>(const GemmParams&, cudaStream_t);
#define RACB_GEMM_EXTERN_TMA(MODE, ITERS, LAYOUT, V) \
    extern template int launch_inst<MODE, ITERS, LAYOUT, V, true, true>(const GemmParams&, cudaStream_t);

}  // namespace racb
