// gemm_noalloc.cu -- the split-K GEMM for callers that must not allocate.
//
// rac_gemm_async takes the split-K partial sums from a workspace that it
// allocates on the caller's stream.  Some callers cannot let a library do
// that: hosts that hand each plugin a fixed device-memory budget and account
// for every byte (an allocation inside the library breaks that accounting and
// can fail under memory pressure in the middle of a step), and
// latency-critical callers for whom a device allocation is a possible stall.
// For them, rac_gemm_splitk_noalloc_async runs the same kernels with the
// partial sums in a fixed array compiled into this library, so the call
// allocates nothing: no cudaMalloc, cudaMallocAsync, cudaFree or allocating
// library routine is reached from it.
//
// The price: every GPU that loads the library holds the array (kScratchBytes)
// until the process exits, problems needing more than that are rejected, and
// all calls share it -- calls whose kernels overlap on the GPU (two streams,
// or two host threads) race on it.
#include <cstdio>
#include <mutex>

#include "gemm_kernel.cuh"
#include "rac_b200.h"
#include "rac_internal.h"

#define RAC_API extern "C" __attribute__((visibility("default")))

namespace racb {
namespace {

// 16 MiB of partial sums: splits * M * N floats.  The BASELINE skinny shape
// (M=16, N=11008, 7 splits) needs 4.9 MiB.
constexpr size_t kScratchFloats = size_t(4) << 20;
constexpr size_t kScratchBytes = kScratchFloats * sizeof(float);

static __device__ __align__(256) float g_splitk_scratch[kScratchFloats];

// Device address of g_splitk_scratch per device.  In host code the symbol is
// only a host-side stand-in: passing it to a kernel would fault or touch the
// wrong memory, so the device address is fetched once per device, with that
// device current, by cudaGetSymbolAddress.
float* g_scratch_addr[64] = {};
cudaError_t g_scratch_err[64] = {};
std::once_flag g_scratch_once[64];

int scratch_for_current_device(float** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) { cudaGetLastError(); return kErrCuda; }
    if (dev < 0 || dev >= 64) return kErrUnsupported;
    std::call_once(g_scratch_once[dev], [dev] {
        void* p = nullptr;
        g_scratch_err[dev] = cudaGetSymbolAddress(&p, g_splitk_scratch);
        if (g_scratch_err[dev] == cudaSuccess) g_scratch_addr[dev] = static_cast<float*>(p);
        else cudaGetLastError();
    });
    if (g_scratch_err[dev] != cudaSuccess || !g_scratch_addr[dev]) return kErrCuda;
    *out = g_scratch_addr[dev];
    return kOk;
}

}  // namespace
}  // namespace racb

// See include/rac_b200.h.  The first call on a device looks up the array's
// device address (cudaGetSymbolAddress); make that first call before any
// stream capture on that device.  Nothing in the array has to start at zero:
// each split writes every element of its M x N slice before the reduction
// kernel reads it.
RAC_API int rac_gemm_splitk_noalloc_async(const float* A, long long lda, const float* B,
                                          long long ldb, float* C, long long ldc,
                                          const float* Cin, long long ldcin, const float* bias,
                                          int M, int N, int K, int layout, int mode, int iters,
                                          float alpha, float beta, int act, int splits,
                                          void* stream) {
    using namespace racb;
    const char* name = "rac_gemm_splitk_noalloc_async";
    if (iters <= 0) iters = rac_get_cordic_iters();
    if (mode < 0) mode = rac_get_cordic_mode();
    if (iters > kMaxIters) iters = kMaxIters;
    if (!A || !B || !C) return record_status(kErrNullPtr, "rac_gemm_splitk_noalloc_async: null pointer");
    if (M <= 0 || N <= 0 || K <= 0 || splits < 0)
        return record_status(kErrInvalidDim, "rac_gemm_splitk_noalloc_async: invalid dimension");
    if (layout < kNN || layout > kTN || act < kActNone || act > kActSilu ||
        (mode != kFast && mode != kCordic && mode != kShiftAdd))
        return record_status(kErrUnsupported, "rac_gemm_splitk_noalloc_async: unsupported layout/mode/act");
    if (beta != 0.0f && !Cin) Cin = C;

    GemmParams p{};
    p.A = A; p.B = B; p.C = C; p.Cin = Cin ? Cin : C; p.bias = bias;
    p.M = M; p.N = N; p.K = K;
    p.lda = lda; p.ldb = ldb; p.ldc = ldc; p.ldcin = Cin ? ldcin : ldc;
    p.alpha = alpha; p.beta = beta; p.act = act; p.iters = iters;

    int S = splits > 0 ? splits : splitk_count(p, layout, mode, 0);
    if (S > K) S = K;
    p.kchunk = ((K + S - 1) / S + 7) / 8 * 8;            // multiple of the tile's BK
    p.splits = (K + p.kchunk - 1) / p.kchunk;
    const size_t need = (size_t)p.splits * (size_t)M * (size_t)N;
    if (need > kScratchFloats) {
        char msg[256];
        std::snprintf(msg, sizeof msg,
                      "%s: %d splits x %d x %d needs %zu floats of scratch, the fixed array holds %zu "
                      "(%zu MiB); use fewer splits or rac_gemm_async", name, p.splits, M, N, need,
                      kScratchFloats, kScratchBytes >> 20);
        return record_status(kErrInvalidDim, msg);
    }
    float* ws = nullptr;
    int st = scratch_for_current_device(&ws);
    if (st != kOk) return record_status(st, "rac_gemm_splitk_noalloc_async: scratch address lookup failed");
    p.ws = ws;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    st = launch_gemm_into(p, layout, mode, 0, s);
    if (st == kOk) st = launch_splitk_reduce(p, s);
    return record_status(st, st == kOk ? "ok" : "rac_gemm_splitk_noalloc_async: launch failed");
}
