// FAST-mode GEMM on packed FFMA2 with TMA staging (gemm_fast.cuh) instantiations.
#include "gemm_fast.cuh"
namespace racb {
RACB_FAST_TMA_INST(kNN, 1) RACB_FAST_TMA_INST(kTN, 1) RACB_FAST_TMA_INST(kNN, 2) RACB_FAST_TMA_INST(kTN, 2)

// dst[c][r] = src[r][c] for a rows x cols source: 32 x 32 tiles through shared
// memory (padded against bank conflicts), coalesced on both sides.
__global__ void __launch_bounds__(256) k_transpose_f32(const float* __restrict__ src, long long lds,
                                                       float* __restrict__ dst, long long ldd,
                                                       int rows, int cols) {
    __shared__ float t[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;        // 8 rows of 32
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int r = r0 + ty + k, c = c0 + tx;
        if (r < rows && c < cols) t[ty + k][tx] = src[(long long)r * lds + c];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 32; k += 8) {
        const int c = c0 + ty + k, r = r0 + tx;
        if (r < rows && c < cols) dst[(long long)c * ldd + r] = t[tx][ty + k];
    }
}

// FAST NT on the NN TMA kernel over a transposed copy of B (pooled, freed in
// stream order).
int launch_fast_tma_nt(const GemmParams& p_in, cudaStream_t s) {
    if (p_in.ws) return kErrUnsupported;
    // TMA rules for the NN launch: A 16-byte aligned with a 16-byte leading
    // dimension; the transposed B has leading dimension N
    if (p_in.N % 4 != 0 || (reinterpret_cast<uintptr_t>(p_in.A) & 15) || (p_in.lda * 4) % 16)
        return kErrUnsupported;
    GemmParams q;
    keep_device_pool();
    float* bt = nullptr;
    const size_t bytes = sizeof(float) * (size_t)p_in.N * p_in.K;
    if (cudaMallocAsync(reinterpret_cast<void**>(&bt), bytes, s) != cudaSuccess) {
        cudaGetLastError();
        return kErrUnsupported;                        // the general kernel needs no buffer
    }
    dim3 tg((p_in.K + 31) / 32, (p_in.N + 31) / 32);
    int st = kOk;
    if (tg.y > 65535) st = kErrUnsupported;
    else {
        k_transpose_f32<<<tg, 256, 0, s>>>(p_in.B, p_in.ldb, bt, p_in.N, p_in.N, p_in.K);
        if (cudaGetLastError() != cudaSuccess) st = kErrCuda;
    }
    if (st == kOk) {
        q = p_in;
        q.B = bt;
        q.ldb = p_in.N;
        st = launch_fast_tma<kNN, 2>(q, s);
    }
    cudaFreeAsync(bt, s);
    return st;
}
}
