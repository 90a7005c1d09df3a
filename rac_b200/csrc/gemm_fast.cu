// gemm_fast.cu -- FAST-mode GEMM (sign-XOR FMA = plain FFMA) for sm_100a.
//
// FAST is the default mode of the reference's PyTorch layer
// (rac_torch/rac_torch.py:1033); its MAC is one FMA (rac_kernels.hip:56-64),
// so unlike the CORDIC kernel this one is bound by the FMA pipe only if the
// loads and address arithmetic stay out of the issue slots.  It uses the
// paired FP32 instruction of sm_100 (fma.rn.f32x2: two FMAs per issue slot,
// same FMA-pipe throughput) on 2x2 blocks of the register tile:
//   D = (a_i, a_i+1) * (b_j,   b_j+1) + D  -> C[i][j],   C[i+1][j+1]
//   S = (a_i, a_i+1) * (b_j+1, b_j)   + S  -> C[i][j+1], C[i+1][j]
// Each lane is one FMA accumulated over k in ascending order, so the result
// is bit-identical to the sequential restatement, like the other kernels.
//
// 128x128 CTA tile, 256 threads, 8x8 register tile per thread in 4-wide row /
// column groups (conflict-free float4 shared reads), BK = 16, operands staged
// global -> registers -> shared with a double buffer.
#include "gemm_kernel.cuh"

namespace racb {

namespace {

constexpr int FBM = 128, FBN = 128, FBK = 16, FTM = 8, FTN = 8;
constexpr int FTX = FBN / FTN, FTY = FBM / FTM, FNT = FTX * FTY;   // 16 x 16 = 256

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpack2(unsigned long long v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ unsigned long long ffma2(unsigned long long a, unsigned long long b,
                                                    unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

template <int LAYOUT>
__global__ void __launch_bounds__(FNT, 2) k_gemm_fast(const __grid_constant__ GemmParams p) {
    constexpr bool A_KCOLS = (LAYOUT != kTN);
    constexpr bool B_KCOLS = (LAYOUT == kNT);
    __shared__ __align__(16) float As[2][FBK * FBM];
    __shared__ __align__(16) float Bs[2][FBK * FBN];
    const int tid = threadIdx.x;
    const int tx = tid % FTX, ty = tid / FTX;
    const int m0 = blockIdx.x * FBM, n0 = blockIdx.y * FBN;
    auto row_of = [&](int i) { return (i >> 2) * (FBM / 2) + ty * 4 + (i & 3); };
    auto col_of = [&](int j) { return (j >> 2) * (FBN / 2) + tx * 4 + (j & 3); };

    TileLoader<A_KCOLS ? FBM : FBK, A_KCOLS ? FBK : FBM, FNT, true> la;
    TileLoader<B_KCOLS ? FBN : FBK, B_KCOLS ? FBK : FBN, FNT, true> lb;
    auto load_tiles = [&](int k0) {
        if constexpr (A_KCOLS) la.load(p.A, p.lda, m0, k0, p.M, p.K, tid);
        else                   la.load(p.A, p.lda, k0, m0, p.K, p.M, tid);
        if constexpr (B_KCOLS) lb.load(p.B, p.ldb, n0, k0, p.N, p.K, tid);
        else                   lb.load(p.B, p.ldb, k0, n0, p.K, p.N, tid);
    };
    auto store_tiles = [&](int buf) {
        la.template store<A_KCOLS, FBM>(As[buf], tid);
        lb.template store<B_KCOLS, FBN>(Bs[buf], tid);
    };

    // D[ip][jp] holds (C[2ip][2jp], C[2ip+1][2jp+1]); S[ip][jp] holds
    // (C[2ip][2jp+1], C[2ip+1][2jp]) of the thread's 8x8 tile.
    unsigned long long D[4][4], S[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) { D[i][j] = 0ull; S[i][j] = 0ull; }

    const int ktiles = (p.K + FBK - 1) / FBK;
    load_tiles(0);
    store_tiles(0);
    __syncthreads();
    for (int kt = 0; kt < ktiles; ++kt) {
        const int buf = kt & 1;
        if (kt + 1 < ktiles) load_tiles((kt + 1) * FBK);
        const float* __restrict__ Asb = As[buf];
        const float* __restrict__ Bsb = Bs[buf];
#pragma unroll 4
        for (int kk = 0; kk < FBK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&Asb[kk * FBM + row_of(0)]);
            const float4 a1 = *reinterpret_cast<const float4*>(&Asb[kk * FBM + row_of(4)]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bsb[kk * FBN + col_of(0)]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bsb[kk * FBN + col_of(4)]);
            const unsigned long long A2[4] = {pack2(a0.x, a0.y), pack2(a0.z, a0.w),
                                              pack2(a1.x, a1.y), pack2(a1.z, a1.w)};
            const unsigned long long B2[4] = {pack2(b0.x, b0.y), pack2(b0.z, b0.w),
                                              pack2(b1.x, b1.y), pack2(b1.z, b1.w)};
            const unsigned long long Bw[4] = {pack2(b0.y, b0.x), pack2(b0.w, b0.z),
                                              pack2(b1.y, b1.x), pack2(b1.w, b1.z)};
#pragma unroll
            for (int ip = 0; ip < 4; ++ip)
#pragma unroll
                for (int jp = 0; jp < 4; ++jp) {
                    D[ip][jp] = ffma2(A2[ip], B2[jp], D[ip][jp]);
                    S[ip][jp] = ffma2(A2[ip], Bw[jp], S[ip][jp]);
                }
        }
        if (kt + 1 < ktiles) store_tiles(buf ^ 1);
        __syncthreads();
    }

    // Epilogue (rac_kernels.hip:790-797, rac_torch.cu:769-776).
#pragma unroll
    for (int ip = 0; ip < 4; ++ip) {
#pragma unroll
        for (int jp = 0; jp < 4; ++jp) {
            float c[2][2];
            unpack2(D[ip][jp], c[0][0], c[1][1]);
            unpack2(S[ip][jp], c[0][1], c[1][0]);
#pragma unroll
            for (int di = 0; di < 2; ++di) {
                const int gm = m0 + row_of(2 * ip + di);
                if (gm >= p.M) continue;
#pragma unroll
                for (int dj = 0; dj < 2; ++dj) {
                    const int gn = n0 + col_of(2 * jp + dj);
                    if (gn >= p.N) continue;
                    const float acc = c[di][dj];
                    float v;
                    if (p.beta != 0.0f)
                        v = __fmaf_rn(p.alpha, acc, __fmul_rn(p.beta, p.Cin[(long long)gm * p.ldcin + gn]));
                    else
                        v = __fmul_rn(p.alpha, acc);
                    if (p.bias) v = __fadd_rn(v, p.bias[gn]);
                    if (p.act) v = apply_act(v, p.act);
                    p.C[(long long)gm * p.ldc + gn] = v;
                }
            }
        }
    }
}

}  // namespace

// FAST-mode GEMM with the paired-FMA kernel: whole-K launches (no split-K),
// vector-aligned operands.  Returns kErrUnsupported otherwise (the caller
// then takes the general kernel).
int launch_gemm_fast(const GemmParams& p, int layout, cudaStream_t s) {
    if (p.ws) return kErrUnsupported;
    dim3 grid((p.M + FBM - 1) / FBM, (p.N + FBN - 1) / FBN);
    if (grid.y > 65535) return kErrInvalidDim;
    switch (layout) {
        case kNN: k_gemm_fast<kNN><<<grid, FNT, 0, s>>>(p); break;
        case kNT: k_gemm_fast<kNT><<<grid, FNT, 0, s>>>(p); break;
        case kTN: k_gemm_fast<kTN><<<grid, FNT, 0, s>>>(p); break;
        default: return kErrUnsupported;
    }
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace racb
