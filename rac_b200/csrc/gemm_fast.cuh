// gemm_fast.cuh -- the FAST-mode GEMM (sign-XOR FMA, rac_kernels.hip:56-64 and
// the FAST branch of rac_fma_iters, :204-211) issued as packed FP32 FMAs.
//
// (a ^ sign b) * |b| is bit-identical to a * b, so each MAC is one fused
// multiply-add, and each output accumulates sequentially over k exactly as
// the reference kernels do.  The general kernel (gemm_kernel.cuh) issues one
// FFMA per MAC plus shared-memory loads, global->register->shared staging and
// loop overhead, which left the FP32 pipe 63 % busy at 81 % issue activity
// (ncu, 4096^3, 44.8 TFLOP/s).  Two changes lift it:
//  * Blackwell's FFMA2 (__ffma2_rn: two independent FMAs on a register pair,
//    each rounded once -- the same bits as two FFMAs) halves the issue slots
//    the MACs take, so the other instructions fit in the FP32 pipe's shadow;
//  * TMA staging through a 4-deep mbarrier ring takes the global loads off the
//    compute warps (with FFMA2 alone, register staging left the kernel
//    waiting on global loads: 3.1-3.4 ms at 4096^3).
// Measured at 4096^3 NN: 2.37 ms, 58.1 TFLOP/s (0.78 of the FP32 FMA peak;
// cuBLAS SGEMM 63.4 TFLOP/s on the same GPU).
#pragma once
#include <atomic>

#include "gemm_kernel.cuh"

namespace racb {

// TMA-staged FAST kernel for the NN and TN layouts: the operand tiles land in
// shared memory through a STAGES-deep ring of cp.async.bulk.tensor copies (no
// multicast; one elected thread issues a stage, every thread waits on the
// stage's mbarrier with a bounded poll, as in k_gemm), so no register or
// instruction of the compute warps is spent on staging and global-load
// latency is hidden by the ring instead of by occupancy.  The tiles land as
// they lie in global memory: NN gives A[m][k] and B[k][n], TN gives A[k][m]
// and B[k][n].  Each k-step is 32 FFMA2 on a thread's 8 x 8 tile, with the
// accumulators paired along n: B pairs come straight from 128-bit loads, A
// values are broadcast into (a, a) pairs.
template <int LAYOUT, int BM, int BN, int BK, int TM, int TN, int STAGES, int MINB>
__global__ void __launch_bounds__((BM / TM) * (BN / TN), MINB)
k_gemm_fast_tma(const __grid_constant__ GemmParams p) {
    static_assert(LAYOUT != kNT, "NT tiles land n-major; the register-staged kernels serve NT");
    static_assert(BK % 2 == 0 && TM % 4 == 0 && TN % 4 == 0, "tile shape");
    constexpr int TX = BN / TN, TY = BM / TM;
    constexpr bool A_MK = (LAYOUT == kNN);             // As[m][k]; TN: As[k][m]
    extern __shared__ __align__(128) float fsm[];
    float* As = fsm;                                   // STAGES x BM*BK
    float* Bs = fsm + STAGES * BM * BK;                // STAGES x BK*BN, Bs[k][n]
    __shared__ __align__(8) uint64_t full_bar[STAGES];

    const int tid = threadIdx.x;
    const int tx = tid % TX, ty = tid / TX;
    // A[m][k]: a thread's rows are TY apart, so the two ty of a warp read
    // adjacent 64-byte rows (different banks); A[k][m]: 4-row groups as in k_gemm.
    auto row_of = [&](int i) {
        if constexpr (A_MK) return i * TY + ty;
        else return (i >> 2) * (BM / (TM / 4)) + ty * 4 + (i & 3);
    };
    auto col_of = [&](int j) { return (j >> 2) * (BN / (TN / 4)) + tx * 4 + (j & 3); };
    const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
    const int ktiles = (p.K + BK - 1) / BK;

    float2 acc[TM][TN / 2];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN / 2; ++j) acc[i][j] = make_float2(0.0f, 0.0f);

    constexpr uint32_t kStageBytes = sizeof(float) * (BM + BN) * BK;
    auto issue = [&](int st, int k0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&full_bar[st], kStageBytes + p.tma_extra_tx);
        if constexpr (A_MK) tma_load_2d(As + st * BM * BK, &p.tmA, k0, m0, &full_bar[st]);
        else                tma_load_2d(As + st * BM * BK, &p.tmA, m0, k0, &full_bar[st]);
        tma_load_2d(Bs + st * BK * BN, &p.tmB, n0, k0, &full_bar[st]);
    };
    if (tid == 0) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) mbar_init(&full_bar[st], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (tid == 0)
        for (int st = 0; st < STAGES && st < ktiles; ++st) issue(st, st * BK);
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
        const float* Ast = As + st * BM * BK;
        const float* Bst = Bs + st * BK * BN;
#pragma unroll
        for (int kk = 0; kk < BK; kk += 2) {
            float2 a01[TM];                            // (a[k], a[k+1]) per row
            if constexpr (A_MK) {
#pragma unroll
                for (int i = 0; i < TM; ++i)
                    a01[i] = *reinterpret_cast<const float2*>(&Ast[row_of(i) * BK + kk]);
            } else {
#pragma unroll
                for (int i = 0; i < TM; i += 4) {
                    const float4 v0 = *reinterpret_cast<const float4*>(&Ast[kk * BM + row_of(i)]);
                    const float4 v1 = *reinterpret_cast<const float4*>(&Ast[(kk + 1) * BM + row_of(i)]);
                    a01[i] = make_float2(v0.x, v1.x);     a01[i + 1] = make_float2(v0.y, v1.y);
                    a01[i + 2] = make_float2(v0.z, v1.z); a01[i + 3] = make_float2(v0.w, v1.w);
                }
            }
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
                float2 b[TN / 2];
#pragma unroll
                for (int j = 0; j < TN; j += 4) {
                    const float4 v = *reinterpret_cast<const float4*>(&Bst[(kk + s2) * BN + col_of(j)]);
                    b[j / 2] = make_float2(v.x, v.y);
                    b[j / 2 + 1] = make_float2(v.z, v.w);
                }
#pragma unroll
                for (int i = 0; i < TM; ++i) {
                    const float av = s2 ? a01[i].y : a01[i].x;
                    const float2 ad = make_float2(av, av);
#pragma unroll
                    for (int j = 0; j < TN / 2; ++j) acc[i][j] = __ffma2_rn(ad, b[j], acc[i][j]);
                }
            }
        }
        __syncthreads();                               // every thread is done with stage st
        if (tid == 0 && !timed_out && kt + STAGES < ktiles) issue(st, (kt + STAGES) * BK);
    }
    if (timed_out && p.err) atomicOr(p.err, 2u);
    store_tile<TM, TN>(p, m0, n0,
                       [&](int i, int j) { return (j & 1) ? acc[i][j >> 1].y : acc[i][j >> 1].x; },
                       row_of, col_of);
}

// TMA tile shapes of the FAST kernel: 1: 128 x 128 x 16, 256 threads, 4 stages
// (64 KB), 2 CTAs per SM -- 2.53-2.56 ms at 4096^3; 2 (the default): 64 x 128 x
// 32, 128 threads, 3 stages (72 KB), 3 CTAs per SM -- 2.37 ms (58.1 TFLOP/s;
// 8192^3: 59.4).  Also measured: 64 x 128 x 16 with 4 stages 2.44-2.47 ms,
// 128 x 128 x 16 with 3 stages 2.53, 128 x 64 x 16 with 4 stages 2.45.
template <int V> struct FastTmaCfg;
template <> struct FastTmaCfg<1> { static constexpr int BM = 128, BN = 128, BK = 16, TM = 8, TN = 8, ST = 4, MINB = 2; };
template <> struct FastTmaCfg<2> { static constexpr int BM = 64, BN = 128, BK = 32, TM = 8, TN = 8, ST = 3, MINB = 3; };


template <int LAYOUT, int V>
int launch_fast_tma(const GemmParams& p_in, cudaStream_t s) {
    using T = FastTmaCfg<V>;
    constexpr int NT = (T::BM / T::TM) * (T::BN / T::TN);
    constexpr int SMEM = T::ST * (T::BM + T::BN) * T::BK * (int)sizeof(float);
    GemmParams p = p_in;
    if (p.ws || !make_tensor_maps(p, LAYOUT, T::BM, T::BN, T::BK)) return kErrUnsupported;
    auto kern = k_gemm_fast_tma<LAYOUT, T::BM, T::BN, T::BK, T::TM, T::TN, T::ST, T::MINB>;
    static std::atomic<bool> attr[64] = {};          // per device; setting it twice is harmless
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return kErrUnsupported;
    if (!attr[dev].load(std::memory_order_acquire)) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
            return kErrCuda;
        attr[dev].store(true, std::memory_order_release);
    }
    dim3 grid((p.M + T::BM - 1) / T::BM, (p.N + T::BN - 1) / T::BN, 1);
    if (grid.y > 65535) return kErrInvalidDim;
    kern<<<grid, NT, SMEM, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

#define RACB_FAST_TMA_INST(LAYOUT, V) template int launch_fast_tma<LAYOUT, V>(const GemmParams&, cudaStream_t);
#define RACB_FAST_TMA_EXTERN(LAYOUT, V) extern template int launch_fast_tma<LAYOUT, V>(const GemmParams&, cudaStream_t);

// NT (B = an nn.Linear weight [N, K]): its tiles would land n-major, where the
// FFMA2 pairs along n cost a register move per pair; a TMA kernel on 128-byte
// swizzled k-major tiles measured 32.5 TFLOP/s at 4096^3 against 37.3 for the
// general kernel.  Instead B is transposed once per call into a pooled buffer
// (2 x |B| bytes of traffic, ~0.3 % of the GEMM at the RACLinear shapes) and
// the NN kernel runs on it -- the same fma sequence per output, so the same bits.
__global__ void k_transpose_f32(const float* __restrict__ src, long long lds, float* __restrict__ dst,
                                long long ldd, int rows, int cols);
int launch_fast_tma_nt(const GemmParams& p_in, cudaStream_t s);

}  // namespace racb
