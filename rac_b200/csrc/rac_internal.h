// rac_internal.h -- declarations shared by the .cu files of librac_b200.so.
// Nothing here is part of the public C ABI (that is include/rac.h and
// include/rac_b200.h).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace racb {

enum Layout : int { kNN = 0, kNT = 1, kTN = 2 };
enum Mode : int { kFast = 0, kCordic = 1, kShiftAdd = 2 };
// kActSwiGLU pairs adjacent output columns: C[m, c] = silu(v[m, 2c]) * v[m, 2c+1]
// (C has N/2 columns) -- the gated FFN's gate and up projections as one GEMM
// over row-interleaved weights.
enum Act : int { kActNone = 0, kActRelu = 1, kActGelu = 2, kActSilu = 3, kActSwiGLU = 4 };

// Status codes: lib/c/rac_cpu.h:54-59 plus the GPU-side ones.
enum Status : int {
    kOk = 0,
    kErrNullPtr = -1,
    kErrInvalidDim = -2,
    kErrAlloc = -3,
    kErrCuda = -4,
    kErrUnsupported = -5,
    kErrDevice = -6,      // a kernel reported a bounded-loop overrun
    kErrNoScratch = -7,
};

struct GemmParams {
    const float* A;
    const float* B;
    float* C;
    const float* Cin;     // read when beta != 0 (may alias C)
    const float* bias;    // [N] or nullptr
    int M, N, K;
    long long lda, ldb, ldc, ldcin;
    float alpha, beta;
    int act;
    int iters;            // CORDIC iteration count (runtime-iteration kernels)
    float k_inv;          // 1/K(iters)
    float coef[24];       // d_i * 2^-i (runtime-iteration kernels)
    // Split-K: when ws != nullptr, CTA z accumulates k in [z*kchunk, (z+1)*kchunk)
    // and stores its raw partial sums to ws[z][M][N]; a second kernel sums the
    // partials in z order and applies the epilogue.
    float* ws;
    int kchunk;
    int splits;
    // TMA-staged kernels: 2-D tensor maps of A and B (built by make_tensor_maps)
    // and the device error word their bounded waits report to.
    alignas(64) CUtensorMap tmA;
    alignas(64) CUtensorMap tmB;
    unsigned int* err;
    unsigned int tma_wait_limit;   // polls of a stage barrier before giving up
    unsigned int tma_extra_tx;     // test hook: bytes expected beyond the copies (0)
};

// Fills p.tmA / p.tmB for a TMA-staged launch with a BM x BN x BK tile.
// Returns false when the operands do not meet the TMA rules (16-byte aligned
// bases and leading dimensions) or the driver entry point is unavailable.
bool make_tensor_maps(GemmParams& p, int layout, int BM, int BN, int BK);
// A 2-D fp32 tensor map (inner dim contiguous, rows ld floats apart) with a
// box_inner x box_outer box; swizzle128 selects the 128-byte swizzle.
bool encode_tensor_2d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer,
                      long long ld, uint32_t box_inner, uint32_t box_outer, bool swizzle128);

// launch_gemm without the split-K decision: launches the tile kernel for p
// as given (p.ws == nullptr: whole K per CTA).
int launch_gemm_into(const GemmParams& p, int layout, int mode, int variant,
                     cudaStream_t stream);
// Sums ws[0..splits-1][M][N] in order and applies the GEMM epilogue of p.
int launch_splitk_reduce(const GemmParams& p, cudaStream_t stream);
// Number of K splits launch_gemm uses for this problem (1 = none).
int splitk_count(const GemmParams& p, int layout, int mode, int variant);

// Launches one GEMM on `stream`. variant 0 = automatic tile choice; the other
// values select a fixed tile (used by the tile sweep in the benchmark).
// Returns a Status; never synchronises.
int launch_gemm(const GemmParams& p, int layout, int mode, int variant,
                cudaStream_t stream);

// Makes the current device's default stream-ordered pool keep freed memory
// (release threshold = max) so that workspaces and staging buffers are not
// re-mapped on every call.  Idempotent, once per device.
void keep_device_pool();

// Records `st` as this thread's rac_last_error() with message `msg`.
int record_status(int st, const char* msg);

// Per-device error word that bounded device loops set (see rac_device.cuh).
unsigned int* device_error_word(int device);

}  // namespace racb
