// shim.cu -- the C ABI of librac_b200.so (include/rac.h, include/rac_b200.h).
//
// Blocking rac.h entry points accept host or device pointers: device (or
// managed) memory is used in place; host memory is staged through
// stream-ordered device allocations on a per-thread, per-device stream.
// Every call records a thread-local status (rac_last_error) and never
// aborts.  There is no CPU path: without a device the call fails with
// RAC_ERR_CUDA.
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "rac_device.cuh"
#include "rac_internal.h"
#include "stream_ops.h"
#include "rac_b200.h"

#define RAC_API extern "C" __attribute__((visibility("default")))

namespace {

using namespace racb;

thread_local int t_status = 0;
thread_local char t_msg[256] = "ok";

int set_status(int st, const char* what) {
    t_status = st;
    if (st == 0) {
        std::snprintf(t_msg, sizeof t_msg, "ok");
    } else {
        const char* kind = st == kErrNullPtr ? "null pointer" : st == kErrInvalidDim ? "invalid dimension"
                         : st == kErrAlloc ? "allocation failed" : st == kErrCuda ? "CUDA error"
                         : st == kErrUnsupported ? "unsupported" : st == kErrDevice ? "device loop limit"
                         : "error";
        cudaError_t ce = cudaGetLastError();
        std::snprintf(t_msg, sizeof t_msg, "%s: %s%s%s", what, kind,
                      ce != cudaSuccess ? " / " : "", ce != cudaSuccess ? cudaGetErrorString(ce) : "");
    }
    return st;
}

std::atomic<int> g_iters{-1};
std::atomic<int> g_mode{-1};

int clamp_gemm_iters(int n) { return n < 1 ? 1 : (n > kMaxIters ? kMaxIters : n); }

void init_knobs() {
    if (g_iters.load() < 0) {
        int it = kDefaultIters;
        if (const char* e = std::getenv("RAC_CORDIC_ITERS")) { int v = std::atoi(e); if (v > 0) it = clamp_gemm_iters(v); }
        int expected = -1;
        g_iters.compare_exchange_strong(expected, it);
    }
    if (g_mode.load() < 0) {
        int m = kCordic;
        if (const char* e = std::getenv("RAC_CORDIC_MODE")) {
            if (!std::strcmp(e, "fast") || !std::strcmp(e, "0")) m = kFast;
            if (!std::strcmp(e, "shiftadd") || !std::strcmp(e, "2")) m = kShiftAdd;
        }
        int expected = -1;
        g_mode.compare_exchange_strong(expected, m);
    }
}

int device_ready(int* dev_out) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) { cudaGetLastError(); return kErrCuda; }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
    if (dev_out) *dev_out = dev;
    return kOk;
}

// Per-thread, per-device stream for blocking calls.
cudaStream_t call_stream(int dev) {
    thread_local std::vector<cudaStream_t> streams;
    if ((int)streams.size() <= dev) streams.resize(dev + 1, nullptr);
    if (!streams[dev]) cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking);
    return streams[dev];
}

bool is_device_ptr(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) { cudaGetLastError(); return false; }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

// One staged buffer of a blocking call.
struct Buf {
    const void* user = nullptr;
    void* dev = nullptr;
    size_t bytes = 0;
    bool staged = false;
    bool out = false;
};

// Scope of a blocking call: stages inputs in, outputs back, frees, syncs.
struct Call {
    int dev = 0;
    cudaStream_t s = nullptr;
    std::vector<Buf> bufs;
    int st = kOk;

    int begin() {
        st = device_ready(&dev);
        if (st == kOk) keep_device_pool();
        if (st == kOk) s = call_stream(dev);
        if (st == kOk && !s) st = kErrCuda;
        return st;
    }
    // in: copy host data to the device; out: copy back at finish.
    void* map(const void* p, size_t bytes, bool in, bool out) {
        if (st != kOk || !p) return const_cast<void*>(p);
        if (bytes == 0 || is_device_ptr(p)) return const_cast<void*>(p);
        Buf b;
        b.user = p; b.bytes = bytes; b.staged = true; b.out = out;
        if (cudaMallocAsync(&b.dev, bytes, s) != cudaSuccess) { st = kErrAlloc; return nullptr; }
        if (in && cudaMemcpyAsync(b.dev, p, bytes, cudaMemcpyHostToDevice, s) != cudaSuccess) st = kErrCuda;
        bufs.push_back(b);
        return b.dev;
    }
    int finish(int launch_status, bool check_loops) {
        if (st == kOk) st = launch_status;
        for (auto& b : bufs) {
            if (st == kOk && b.out &&
                cudaMemcpyAsync(const_cast<void*>(b.user), b.dev, b.bytes, cudaMemcpyDeviceToHost, s) != cudaSuccess)
                st = kErrCuda;
            cudaFreeAsync(b.dev, s);
        }
        if (s && cudaStreamSynchronize(s) != cudaSuccess && st == kOk) st = kErrCuda;
        if (st == kOk && check_loops) {
            unsigned int* w = device_error_word(dev);
            unsigned int h = 0;
            if (w && cudaMemcpy(&h, w, sizeof h, cudaMemcpyDeviceToHost) == cudaSuccess && h) {
                cudaMemset(w, 0, sizeof h);
                st = kErrDevice;
            }
        }
        return st;
    }
};

}  // namespace

namespace racb {
// Lets other translation units of the library record a status with their
// own message (see rac_internal.h).
int record_status(int st, const char* msg) {
    t_status = st;
    std::snprintf(t_msg, sizeof t_msg, "%s", msg ? msg : (st ? "error" : "ok"));
    return st;
}
}  // namespace racb

// ── 1. errors and knobs ─────────────────────────────────────────────────

RAC_API int rac_last_error(void) { return t_status; }
RAC_API const char* rac_last_error_string(void) { return t_msg; }
RAC_API void rac_clear_error(void) { set_status(0, ""); }

RAC_API void rac_set_cordic_iters(int iters) {
    // rac_torch_bind.cpp:205-212: <= 0 resets to the default, else clamp [1, 24].
    init_knobs();
    g_iters.store(iters <= 0 ? kDefaultIters : clamp_gemm_iters(iters));
}
RAC_API int rac_get_cordic_iters(void) { init_knobs(); return g_iters.load(); }
RAC_API void rac_set_cordic_mode(int mode) {
    // rac_torch_bind.cpp:216-219: out-of-range modes fall back to FAST.
    init_knobs();
    g_mode.store((mode == kCordic || mode == kShiftAdd) ? mode : kFast);
}
RAC_API int rac_get_cordic_mode(void) { init_knobs(); return g_mode.load(); }

RAC_API const char* rac_b200_version(void) { return "rac_b200 0.1 (sm_100a)"; }
RAC_API int rac_b200_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) { cudaGetLastError(); return 0; }
    return n;
}
RAC_API void rac_b200_cordic_gemm_directions(int out[24]) {
    if (!out) return;
    for (int i = 0; i < 24; ++i) out[i] = gemm_dir(i);
}

// ── 3. stream-ordered device entry points ───────────────────────────────

static cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

RAC_API int rac_gemm_async(const float* A, long long lda, const float* B, long long ldb,
                           float* C, long long ldc, const float* Cin, long long ldcin,
                           const float* bias, int M, int N, int K, int layout, int mode,
                           int iters, float alpha, float beta, int act, int variant,
                           void* stream) {
    init_knobs();
    if (iters <= 0) iters = g_iters.load();
    if (mode < 0) mode = g_mode.load();
    GemmParams p{};
    p.A = A; p.B = B; p.C = C; p.Cin = Cin ? Cin : C; p.bias = bias;
    p.M = M; p.N = N; p.K = K;
    p.lda = lda; p.ldb = ldb; p.ldc = ldc; p.ldcin = Cin ? ldcin : ldc;
    p.alpha = alpha; p.beta = beta; p.act = act;
    p.iters = clamp_gemm_iters(iters);
    if (act < kActNone || act > kActSwiGLU) return set_status(kErrUnsupported, "rac_gemm_async");
    if (M == 0 || N == 0) return set_status(kOk, "rac_gemm_async");
    return set_status(launch_gemm(p, layout, mode, variant, as_stream(stream)), "rac_gemm_async");
}

static void launch_layout(const float* A, const float* B, float* C, int M, int N, int K,
                          float alpha, float beta, int iters, int mode, void* stream,
                          int layout, const char* name) {
    // Contiguous row-major operands, as in rac_kernels.hip:822-883.
    const long long lda = layout == kTN ? M : K;
    const long long ldb = layout == kNT ? K : N;
    int st = rac_gemm_async(A, lda, B, ldb, C, N, C, N, nullptr, M, N, K, layout, mode, iters,
                            alpha, beta, kActNone, 0, stream);
    set_status(st, name);
}

RAC_API void rac_launch_nn_iters(const float* A, const float* B, float* C, int M, int N, int K,
                                 float alpha, float beta, int iters, int mode, void* stream) {
    launch_layout(A, B, C, M, N, K, alpha, beta, iters, mode, stream, kNN, "rac_launch_nn_iters");
}
RAC_API void rac_launch_nt_iters(const float* A, const float* B, float* C, int M, int N, int K,
                                 float alpha, float beta, int iters, int mode, void* stream) {
    launch_layout(A, B, C, M, N, K, alpha, beta, iters, mode, stream, kNT, "rac_launch_nt_iters");
}
RAC_API void rac_launch_tn_iters(const float* A, const float* B, float* C, int M, int N, int K,
                                 float alpha, float beta, int iters, int mode, void* stream) {
    launch_layout(A, B, C, M, N, K, alpha, beta, iters, mode, stream, kTN, "rac_launch_tn_iters");
}
// rac_kernels.hip:886-909 defaults: iters 24, FAST.
RAC_API void rac_launch_nn(const float* A, const float* B, float* C, int M, int N, int K,
                           float alpha, float beta, void* stream) {
    launch_layout(A, B, C, M, N, K, alpha, beta, 24, kFast, stream, kNN, "rac_launch_nn");
}
RAC_API void rac_launch_nt(const float* A, const float* B, float* C, int M, int N, int K,
                           float alpha, float beta, void* stream) {
    launch_layout(A, B, C, M, N, K, alpha, beta, 24, kFast, stream, kNT, "rac_launch_nt");
}
RAC_API void rac_launch_tn(const float* A, const float* B, float* C, int M, int N, int K,
                           float alpha, float beta, void* stream) {
    launch_layout(A, B, C, M, N, K, alpha, beta, 24, kFast, stream, kTN, "rac_launch_tn");
}

RAC_API int rac_rotate_batch_async(const float2* v, const float* theta, float2* out, long long n,
                                   int iters, int literal_kinv, void* stream) {
    return set_status(rotate_batch(v, theta, out, n, iters, literal_kinv, as_stream(stream)),
                      "rac_rotate_batch_async");
}
RAC_API int rac_project_batch_async(const float2* v, const float* theta, float* out, long long n,
                                    int iters, void* stream) {
    return set_status(project_batch(v, theta, out, n, iters, as_stream(stream)), "rac_project_batch_async");
}
RAC_API int rac_sincos_batch_async(const float* theta, float* s, float* c, long long n, void* stream) {
    return set_status(sincos_batch(theta, s, c, n, as_stream(stream)), "rac_sincos_batch_async");
}
RAC_API int rac_unary_async(const float* x, float* y, long long n, int op, void* stream) {
    return set_status(unary_batch(x, y, n, op, as_stream(stream)), "rac_unary_async");
}
RAC_API int rac_softmax_async(const float* x, float* y, long long rows, int d, void* stream) {
    return set_status(softmax_rows(x, y, rows, d, as_stream(stream)), "rac_softmax_async");
}
RAC_API int rac_rmsnorm_async(const float* x, float* y, const float* gamma, float eps,
                              long long rows, int d, void* stream) {
    return set_status(rmsnorm_rows(x, y, gamma, eps, rows, d, as_stream(stream)), "rac_rmsnorm_async");
}
RAC_API int rac_layernorm_async(const float* x, float* y, const float* gamma, const float* beta,
                                float eps, long long rows, int d, void* stream) {
    return set_status(layernorm_rows(x, y, gamma, beta, eps, rows, d, as_stream(stream)),
                      "rac_layernorm_async");
}
RAC_API int rac_rope_cache_async(float* cos_out, float* sin_out, int max_seq, int head_dim,
                                 float base, void* stream) {
    return set_status(rope_cache(cos_out, sin_out, max_seq, head_dim, base, as_stream(stream)),
                      "rac_rope_cache_async");
}
RAC_API int rac_rope_apply_async(float* x, const float* cos_tab, const float* sin_tab,
                                 const int* pos, long long batch_heads, int seq, int head_dim,
                                 int form, void* stream) {
    return set_status(rope_apply(x, cos_tab, sin_tab, pos, batch_heads, seq, head_dim, form,
                                 as_stream(stream)), "rac_rope_apply_async");
}
RAC_API int rac_check_device_errors(void* stream) {
    int dev = 0;
    int st = device_ready(&dev);
    if (st != kOk) return set_status(st, "rac_check_device_errors");
    if (cudaStreamSynchronize(as_stream(stream)) != cudaSuccess)
        return set_status(kErrCuda, "rac_check_device_errors");
    unsigned int* w = device_error_word(dev);
    unsigned int h = 0;
    if (!w || cudaMemcpy(&h, w, sizeof h, cudaMemcpyDeviceToHost) != cudaSuccess)
        return set_status(kErrCuda, "rac_check_device_errors");
    if (h) { cudaMemset(w, 0, sizeof h); return set_status(kErrDevice, "rac_check_device_errors"); }
    return set_status(kOk, "rac_check_device_errors");
}

// ── blocking entry points (rac.h and batch forms) ───────────────────────

// rac_matmul with host-resident A and C: the transfers are pipelined with
// the compute.  B goes first; A follows in two row blocks on a copy stream,
// and each block's GEMM starts on the compute stream as soon as its rows have
// landed, while the previous block's C rows travel back.  Two blocks keep
// each launch large enough to fill the SMs (the GEMM's per-SM balance is
// unchanged: 4096 rows -> 2 x 2048).  Each output element's arithmetic does
// not depend on the row blocking, so the result equals one launch's, except
// where a block's shape selects split-K (few output tiles, K >= 1024), whose
// partial sums associate differently.
// Per-thread, per-device upload and download streams of the blocking calls.
struct CopyStreams { cudaStream_t h2d = nullptr, d2h = nullptr; };
static CopyStreams* copy_streams(int dev) {
    thread_local std::vector<CopyStreams> per_dev;
    if ((int)per_dev.size() <= dev) per_dev.resize(dev + 1);
    CopyStreams& ss = per_dev[dev];
    for (cudaStream_t* q : {&ss.h2d, &ss.d2h})
        if (!*q && cudaStreamCreateWithFlags(q, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    return &ss;
}

// One argument of a chunked blocking call.  `unit` bytes per work unit for
// arrays split with the work (vectors, rows, planes); unit == 0 marks an
// array every chunk needs whole (gamma, tables, a mask) of `whole` bytes.
// Device (or managed) pointers are used in place.
struct Arg {
    const void* host;
    size_t unit, whole;
    bool in, out;
    char* dev = nullptr;
    bool staged = false;
};

// Runs launch(u0, u1, stream) over [0, units) in chunks: with host arrays the
// upload of chunk i+1 (one stream), the kernel of chunk i (the call stream)
// and the download of chunk i-1 (another stream; PCIe is full duplex)
// overlap.  Work units are independent, so chunking does not change any
// result.  `align` keeps chunk starts on multiples of that many units.
template <class Launch>
static int run_chunked(Call& c, long long units, Arg* args, int nargs, long long align, Launch&& launch) {
    size_t staged_bytes = 0;
    for (int i = 0; i < nargs; ++i) {
        Arg& a = args[i];
        a.staged = a.host && !is_device_ptr(a.host);
        a.dev = const_cast<char*>(static_cast<const char*>(a.host));
        if (a.staged) staged_bytes += a.unit ? a.unit * (size_t)units : a.whole;
    }
    if (staged_bytes == 0) {                     // everything on the device already
        const int st = launch(0LL, units, c.s);
        return st;
    }
    CopyStreams* ss = copy_streams(c.dev);
    if (!ss) return kErrCuda;
    int st = kOk;
    for (int i = 0; i < nargs && st == kOk; ++i) {
        Arg& a = args[i];
        if (!a.staged) continue;
        const size_t bytes = a.unit ? a.unit * (size_t)units : a.whole;
        void* d = nullptr;
        if (cudaMallocAsync(&d, bytes, c.s) != cudaSuccess) { cudaGetLastError(); st = kErrAlloc; break; }
        a.dev = static_cast<char*>(d);
    }
    std::vector<cudaEvent_t> evs;
    auto event = [&]() {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess) evs.push_back(e);
        return e;
    };
    auto chk = [&](cudaError_t e) { if (e != cudaSuccess && st == kOk) st = kErrCuda; };
    if (st == kOk) {
        cudaEvent_t ev_alloc = event();
        chk(cudaEventRecord(ev_alloc, c.s));
        chk(cudaStreamWaitEvent(ss->h2d, ev_alloc, 0));
        chk(cudaStreamWaitEvent(ss->d2h, ev_alloc, 0));
        for (int i = 0; i < nargs; ++i)          // whole arrays first
            if (args[i].staged && args[i].in && !args[i].unit)
                chk(cudaMemcpyAsync(args[i].dev, args[i].host, args[i].whole, cudaMemcpyHostToDevice, ss->h2d));
        // ~8 MiB of staged traffic per chunk, at most 16 chunks.
        long long chunks = (long long)(staged_bytes >> 23);
        chunks = chunks < 1 ? 1 : (chunks > 16 ? 16 : chunks);
        long long per = (units + chunks - 1) / chunks;
        per = (per + align - 1) / align * align;
        for (long long u0 = 0; u0 < units && st == kOk; u0 += per) {
            const long long u1 = u0 + per < units ? u0 + per : units;
            for (int i = 0; i < nargs; ++i) {
                const Arg& a = args[i];
                if (a.staged && a.in && a.unit)
                    chk(cudaMemcpyAsync(a.dev + a.unit * u0, static_cast<const char*>(a.host) + a.unit * u0,
                                        a.unit * (u1 - u0), cudaMemcpyHostToDevice, ss->h2d));
            }
            cudaEvent_t in = event();
            chk(cudaEventRecord(in, ss->h2d));
            chk(cudaStreamWaitEvent(c.s, in, 0));
            if (st == kOk) st = launch(u0, u1, c.s);
            cudaEvent_t done = event();
            chk(cudaEventRecord(done, c.s));
            chk(cudaStreamWaitEvent(ss->d2h, done, 0));
            for (int i = 0; i < nargs; ++i) {
                const Arg& a = args[i];
                if (a.staged && a.out && a.unit)
                    chk(cudaMemcpyAsync(const_cast<char*>(static_cast<const char*>(a.host)) + a.unit * u0,
                                        a.dev + a.unit * u0, a.unit * (u1 - u0), cudaMemcpyDeviceToHost, ss->d2h));
            }
        }
        for (cudaStream_t q : {ss->h2d, ss->d2h}) {   // frees after the copies' last use
            cudaEvent_t e = event();
            chk(cudaEventRecord(e, q));
            chk(cudaStreamWaitEvent(c.s, e, 0));
        }
    }
    for (int i = 0; i < nargs; ++i)
        if (args[i].staged && args[i].dev) cudaFreeAsync(args[i].dev, c.s);
    if (cudaStreamSynchronize(c.s) != cudaSuccess && st == kOk) st = kErrCuda;
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
    return st;
}

static int sm_count_of(int dev) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) {
        cudaGetLastError();
        sms = 148;
    }
    return sms;
}

// Blocking rac_matmul with host A and C (and B on the host or the device):
// C is computed in R row blocks so that copies overlap compute.  One stream
// uploads B and then every row block of A; the compute stream runs each
// block's GEMM as soon as its rows have landed; a third stream downloads each
// C block as soon as it is done (PCIe is full duplex), so only B, the first
// A block and the last C block are not hidden behind compute.  The caller
// uses this path only when the whole problem would not split K, and the
// blocks never split either, so every output is one GEMM over the whole of
// K and the bits equal a single launch's.
static int matmul_pipelined(Call& c, const float* A, const float* B, bool b_host, float* C, int M,
                            int N, int K, int iters, int mode) {
    CopyStreams* css = copy_streams(c.dev);
    if (!css) return kErrCuda;
    CopyStreams& ss = *css;

    float* dA = nullptr;
    float* dB = nullptr;
    float* dC = nullptr;
    bool alloc_ok = cudaMallocAsync(reinterpret_cast<void**>(&dA), sizeof(float) * (size_t)M * K, c.s) == cudaSuccess &&
                    cudaMallocAsync(reinterpret_cast<void**>(&dC), sizeof(float) * (size_t)M * N, c.s) == cudaSuccess;
    if (alloc_ok && b_host)
        alloc_ok = cudaMallocAsync(reinterpret_cast<void**>(&dB), sizeof(float) * (size_t)K * N, c.s) == cudaSuccess;
    if (!alloc_ok) {
        cudaGetLastError();
        if (dA) cudaFreeAsync(dA, c.s);
        if (dC) cudaFreeAsync(dC, c.s);
        return kErrAlloc;
    }

    // Four row blocks when each still fills the SMs several times over with
    // 64 x 64 tiles, else two.
    const long long block_tiles = (long long)((M / 4 + 63) / 64) * ((N + 63) / 64);
    const int R = block_tiles >= 4LL * sm_count_of(c.dev) ? 4 : 2;
    int rb[5];
    for (int r = 0; r <= R; ++r) rb[r] = (int)((long long)M * r / R);

    std::vector<cudaEvent_t> evs;
    auto event = [&]() {
        cudaEvent_t e = nullptr;
        if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) == cudaSuccess) evs.push_back(e);
        return e;
    };
    int st = kOk;
    auto chk = [&](cudaError_t e) { if (e != cudaSuccess && st == kOk) st = kErrCuda; };

    // Copy streams start after the allocations exist.
    cudaEvent_t ev_alloc = event();
    chk(cudaEventRecord(ev_alloc, c.s));
    for (cudaStream_t q : {ss.h2d, ss.d2h}) chk(cudaStreamWaitEvent(q, ev_alloc, 0));
    if (b_host)
        chk(cudaMemcpyAsync(dB, B, sizeof(float) * (size_t)K * N, cudaMemcpyHostToDevice, ss.h2d));
    cudaEvent_t ev_a[4];
    for (int r = 0; r < R; ++r) {
        const size_t off = (size_t)rb[r] * K;
        if (rb[r + 1] > rb[r])
            chk(cudaMemcpyAsync(dA + off, A + off, sizeof(float) * (size_t)(rb[r + 1] - rb[r]) * K,
                                cudaMemcpyHostToDevice, ss.h2d));
        ev_a[r] = event();
        chk(cudaEventRecord(ev_a[r], ss.h2d));
    }

    GemmParams p{};
    p.B = b_host ? dB : B;
    p.N = N; p.K = K; p.lda = K; p.ldb = N; p.ldc = N; p.ldcin = N;
    p.alpha = 1.0f; p.beta = 0.0f;
    p.iters = iters;
    for (int r = 0; r < R && st == kOk; ++r) {
        if (rb[r + 1] <= rb[r]) continue;
        chk(cudaStreamWaitEvent(c.s, ev_a[r], 0));
        p.A = dA + (size_t)rb[r] * K;
        p.C = dC + (size_t)rb[r] * N;
        p.Cin = p.C;
        p.M = rb[r + 1] - rb[r];
        p.ws = nullptr; p.splits = 1; p.kchunk = 0;
        if (st == kOk) st = launch_gemm_into(p, kNN, mode, 0, c.s);
        cudaEvent_t done = event();
        chk(cudaEventRecord(done, c.s));
        chk(cudaStreamWaitEvent(ss.d2h, done, 0));
        if (st == kOk)
            chk(cudaMemcpyAsync(C + (size_t)rb[r] * N, p.C, sizeof(float) * (size_t)p.M * N,
                                cudaMemcpyDeviceToHost, ss.d2h));
    }
    // The frees on c.s are ordered after the copy streams' last use.
    for (cudaStream_t q : {ss.h2d, ss.d2h}) {
        cudaEvent_t e = event();
        chk(cudaEventRecord(e, q));
        chk(cudaStreamWaitEvent(c.s, e, 0));
    }
    cudaFreeAsync(dA, c.s);
    cudaFreeAsync(dC, c.s);
    if (dB) cudaFreeAsync(dB, c.s);
    if (cudaStreamSynchronize(c.s) != cudaSuccess && st == kOk) st = kErrCuda;
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
    return st;
}

static int do_matmul(const float* A, const float* B, float* C, int M, int N, int K, int iters,
                     int mode) {
    if (!A || !B || !C) return kErrNullPtr;
    if (M <= 0 || N <= 0 || K <= 0) return kErrInvalidDim;
    Call c;
    if (c.begin() != kOk) return c.st;
    init_knobs();
    iters = clamp_gemm_iters(iters <= 0 ? g_iters.load() : iters);
    mode = mode < 0 ? g_mode.load() : mode;
    const bool host_a = !is_device_ptr(A), host_c = !is_device_ptr(C);
    if (host_a && host_c && M >= 256) {
        GemmParams whole{};
        whole.M = M; whole.N = N; whole.K = K;
        if (splitk_count(whole, kNN, mode, 0) == 1) {
            const int st = matmul_pipelined(c, A, B, !is_device_ptr(B), C, M, N, K, iters, mode);
            return c.finish(st, false);
        }
    }
    const float* dA = (const float*)c.map(A, sizeof(float) * (size_t)M * K, true, false);
    const float* dB = (const float*)c.map(B, sizeof(float) * (size_t)K * N, true, false);
    float* dC = (float*)c.map(C, sizeof(float) * (size_t)M * N, false, true);
    int st = kOk;
    if (c.st == kOk) {
        GemmParams p{};
        p.A = dA; p.B = dB; p.C = dC; p.Cin = dC;
        p.M = M; p.N = N; p.K = K; p.lda = K; p.ldb = N; p.ldc = N; p.ldcin = N;
        p.alpha = 1.0f; p.beta = 0.0f;
        p.iters = iters;
        st = launch_gemm(p, kNN, mode, 0, c.s);
    }
    return c.finish(st, false);
}

RAC_API void rac_matmul(float* A, float* B, float* C, int M, int N, int K) {
    set_status(do_matmul(A, B, C, M, N, K, -1, -1), "rac_matmul");
}
RAC_API void rac_matmul_ex(const float* A, const float* B, float* C, int M, int N, int K,
                           int iters, int mode) {
    set_status(do_matmul(A, B, C, M, N, K, iters, mode), "rac_matmul_ex");
}

static int do_rotate(const float2* v, const float* th, float2* out, long long n, int iters,
                     int literal) {
    if (n < 0) return kErrInvalidDim;
    if (n == 0) return kOk;
    if (!v || !th || !out) return kErrNullPtr;
    Call c;
    if (c.begin() != kOk) return c.st;
    Arg a[3] = {{v, sizeof(float2), 0, true, false}, {th, sizeof(float), 0, true, false},
                {out, sizeof(float2), 0, false, true}};
    const int st = run_chunked(c, n, a, 3, 64, [&](long long u0, long long u1, cudaStream_t s) {
        return rotate_batch(reinterpret_cast<const float2*>(a[0].dev) + u0, reinterpret_cast<const float*>(a[1].dev) + u0,
                            reinterpret_cast<float2*>(a[2].dev) + u0, u1 - u0, iters, literal, s);
    });
    return c.finish(st, true);
}

RAC_API void rac_rotate_batch(float2* v, float* theta, float2* out, int n) {
    set_status(do_rotate(v, theta, out, n, kDefaultIters, 1), "rac_rotate_batch");
}
RAC_API void rac_rotate_batch_n(const float2* v, const float* theta, float2* out, int n, int iters) {
    set_status(do_rotate(v, theta, out, n, iters, 0), "rac_rotate_batch_n");
}
RAC_API float2 rac_rotate(float2 v, float theta) {
    float2 out = make_float2(0.f, 0.f);
    set_status(do_rotate(&v, &theta, &out, 1, kDefaultIters, 1), "rac_rotate");
    return out;
}
RAC_API float2 rac_rotate_precision(float2 v, float theta, int iters) {
    float2 out = make_float2(0.f, 0.f);
    set_status(do_rotate(&v, &theta, &out, 1, iters, 0), "rac_rotate_precision");
    return out;
}

static int do_project(const float2* v, const float* th, float* out, long long n, int iters) {
    if (n < 0) return kErrInvalidDim;
    if (n == 0) return kOk;
    if (!v || !th || !out) return kErrNullPtr;
    Call c;
    if (c.begin() != kOk) return c.st;
    Arg a[3] = {{v, sizeof(float2), 0, true, false}, {th, sizeof(float), 0, true, false},
                {out, sizeof(float), 0, false, true}};
    const int st = run_chunked(c, n, a, 3, 64, [&](long long u0, long long u1, cudaStream_t s) {
        return project_batch(reinterpret_cast<const float2*>(a[0].dev) + u0, reinterpret_cast<const float*>(a[1].dev) + u0,
                             reinterpret_cast<float*>(a[2].dev) + u0, u1 - u0, iters, s);
    });
    return c.finish(st, true);
}
RAC_API void rac_project_batch_n(const float2* v, const float* theta, float* out, int n, int iters) {
    set_status(do_project(v, theta, out, n, iters), "rac_project_batch_n");
}
RAC_API float rac_project_precision(float2 v, float theta, int iters) {
    float out = 0.f;
    set_status(do_project(&v, &theta, &out, 1, iters), "rac_project_precision");
    return out;
}

static int do_unary(const float* x, float* y, long long n, int op) {
    if (n < 0) return kErrInvalidDim;
    if (n == 0) return kOk;
    if (!x || !y) return kErrNullPtr;
    Call c;
    if (c.begin() != kOk) return c.st;
    Arg a[2] = {{x, sizeof(float), 0, true, false}, {y, sizeof(float), 0, false, true}};
    const int st = run_chunked(c, n, a, 2, 64, [&](long long u0, long long u1, cudaStream_t s) {
        return unary_batch(reinterpret_cast<const float*>(a[0].dev) + u0, reinterpret_cast<float*>(a[1].dev) + u0,
                           u1 - u0, op, s);
    });
    return c.finish(st, false);
}
RAC_API void rac_exp_batch(const float* x, float* y, int n) { set_status(do_unary(x, y, n, kUnaryExp), "rac_exp_batch"); }
RAC_API void rac_tanh_batch(const float* x, float* y, int n) { set_status(do_unary(x, y, n, kUnaryTanh), "rac_tanh_batch"); }
RAC_API void rac_rsqrt_batch(const float* x, float* y, int n) { set_status(do_unary(x, y, n, kUnaryRsqrt), "rac_rsqrt_batch"); }
RAC_API void rac_sigmoid_batch(const float* x, float* y, int n) { set_status(do_unary(x, y, n, kUnarySigmoid), "rac_sigmoid_batch"); }
static float unary1(float x, int op, const char* name) {
    float y = 0.f;
    set_status(do_unary(&x, &y, 1, op), name);
    return y;
}
RAC_API float rac_exp(float x) { return unary1(x, kUnaryExp, "rac_exp"); }
RAC_API float rac_tanh(float x) { return unary1(x, kUnaryTanh, "rac_tanh"); }
RAC_API float rac_rsqrt(float x) { return unary1(x, kUnaryRsqrt, "rac_rsqrt"); }
RAC_API float rac_sigmoid(float x) { return unary1(x, kUnarySigmoid, "rac_sigmoid"); }

RAC_API void rac_sincos_batch(const float* theta, float* s, float* c_out, int n) {
    int st = kOk;
    if (n < 0) st = kErrInvalidDim;
    else if (n > 0 && (!theta || !s || !c_out)) st = kErrNullPtr;
    else if (n > 0) {
        Call c;
        if (c.begin() == kOk) {
            Arg a[3] = {{theta, sizeof(float), 0, true, false}, {s, sizeof(float), 0, false, true},
                        {c_out, sizeof(float), 0, false, true}};
            const int r = run_chunked(c, n, a, 3, 64, [&](long long u0, long long u1, cudaStream_t strm) {
                return sincos_batch(reinterpret_cast<const float*>(a[0].dev) + u0, reinterpret_cast<float*>(a[1].dev) + u0,
                                    reinterpret_cast<float*>(a[2].dev) + u0, u1 - u0, strm);
            });
            st = c.finish(r, true);
        } else {
            st = c.st;
        }
    }
    set_status(st, "rac_sincos_batch");
}
RAC_API void rac_sincos(float theta, float* s, float* c) {
    float ls = 0.f, lc = 0.f;
    rac_sincos_batch(&theta, &ls, &lc, 1);
    if (s) *s = ls;
    if (c) *c = lc;
}

static int do_rows(int op, const float* x, float* y, const float* g, const float* b, float eps,
                   long long rows, int d) {
    if (rows < 0 || d <= 0) return kErrInvalidDim;
    if (rows == 0) return kOk;
    if (!x || !y) return kErrNullPtr;
    Call c;
    if (c.begin() != kOk) return c.st;
    const size_t row = sizeof(float) * (size_t)d;
    Arg a[4] = {{x, row, 0, true, false}, {y, row, 0, false, true},
                {g, 0, row, true, false}, {b, 0, row, true, false}};
    const int st = run_chunked(c, rows, a, 4, 1, [&](long long r0, long long r1, cudaStream_t s) {
        const float* dx = reinterpret_cast<const float*>(a[0].dev) + r0 * d;
        float* dy = reinterpret_cast<float*>(a[1].dev) + r0 * d;
        const float* dg = reinterpret_cast<const float*>(a[2].dev);
        const float* db = reinterpret_cast<const float*>(a[3].dev);
        if (op == 0) return softmax_rows(dx, dy, r1 - r0, d, s);
        if (op == 1) return rmsnorm_rows(dx, dy, dg, eps, r1 - r0, d, s);
        return layernorm_rows(dx, dy, dg, db, eps, r1 - r0, d, s);
    });
    return c.finish(st, false);
}
RAC_API void rac_softmax(float* x, float* out, int n) {
    set_status(do_rows(0, x, out, nullptr, nullptr, 0.f, 1, n), "rac_softmax");
}
RAC_API void rac_softmax_batch(const float* x, float* out, int batch, int n) {
    set_status(do_rows(0, x, out, nullptr, nullptr, 0.f, batch, n), "rac_softmax_batch");
}
RAC_API void rac_rmsnorm(const float* x, float* y, const float* gamma, float eps, int rows, int d) {
    set_status(do_rows(1, x, y, gamma, nullptr, eps, rows, d), "rac_rmsnorm");
}
RAC_API void rac_layernorm(const float* x, float* y, const float* gamma, const float* beta,
                           float eps, int rows, int d) {
    set_status(do_rows(2, x, y, gamma, beta, eps, rows, d), "rac_layernorm");
}

static int do_rope_cache(float* cos_out, float* sin_out, int max_seq, int hd, float base) {
    if (!cos_out || !sin_out) return kErrNullPtr;
    if (max_seq <= 0 || hd <= 0 || (hd & 1)) return kErrInvalidDim;
    Call c;
    if (c.begin() != kOk) return c.st;
    const size_t bytes = sizeof(float) * (size_t)max_seq * (hd / 2);
    auto dc = (float*)c.map(cos_out, bytes, false, true);
    auto ds = (float*)c.map(sin_out, bytes, false, true);
    int st = c.st == kOk ? rope_cache(dc, ds, max_seq, hd, base, c.s) : c.st;
    return c.finish(st, true);
}
RAC_API void rac_rope_cache(float* cos_out, float* sin_out, int max_seq, int head_dim, float base) {
    set_status(do_rope_cache(cos_out, sin_out, max_seq, head_dim, base), "rac_rope_cache");
}

static int do_rope_apply(float* x, const float* ct, const float* sn, int batch, int heads, int seq,
                         int hd) {
    if (!x || !ct || !sn) return kErrNullPtr;
    if (batch <= 0 || heads <= 0 || seq <= 0 || hd <= 0 || (hd & 1)) return kErrInvalidDim;
    Call c;
    if (c.begin() != kOk) return c.st;
    const size_t plane = sizeof(float) * (size_t)seq * hd;          // one (batch, head)
    const size_t tb = sizeof(float) * (size_t)seq * (hd / 2);
    Arg a[3] = {{x, plane, 0, true, true}, {ct, 0, tb, true, false}, {sn, 0, tb, true, false}};
    const int st = run_chunked(c, (long long)batch * heads, a, 3, 1,
                               [&](long long p0, long long p1, cudaStream_t s) {
        return rope_apply(reinterpret_cast<float*>(a[0].dev) + p0 * seq * hd, reinterpret_cast<const float*>(a[1].dev),
                          reinterpret_cast<const float*>(a[2].dev), nullptr, p1 - p0, seq, hd, 0, s);
    });
    return c.finish(st, false);
}
RAC_API void rac_rope_apply(float* x, const float* cos_tab, const float* sin_tab, int batch,
                            int n_heads, int seq, int head_dim) {
    set_status(do_rope_apply(x, cos_tab, sin_tab, batch, n_heads, seq, head_dim), "rac_rope_apply");
}

RAC_API int rac_attention_async(const float* q, const float* k, const float* v, const float* mask,
                                int is_causal, float* out, int batch, int n_heads, int seq,
                                int head_dim, void* stream) {
    return set_status(attention(q, k, v, mask, is_causal, out, batch, n_heads, seq, head_dim,
                                as_stream(stream)), "rac_attention_async");
}

static int do_attention(const float* q, const float* k, const float* v, const float* mask,
                        int causal, float* out, int batch, int heads, int seq, int hd) {
    if (!q || !k || !v || !out) return kErrNullPtr;
    if (batch <= 0 || heads <= 0 || seq <= 0 || hd <= 0) return kErrInvalidDim;
    Call c;
    if (c.begin() != kOk) return c.st;
    const size_t plane = sizeof(float) * (size_t)seq * hd;          // one (batch, head)
    Arg a[5] = {{q, plane, 0, true, false}, {k, plane, 0, true, false}, {v, plane, 0, true, false},
                {out, plane, 0, false, true}, {mask, 0, sizeof(float) * (size_t)seq * seq, true, false}};
    const long long planes = (long long)batch * heads;
    // Chunks hold whole batches (align = heads): each runs as (p1 - p0) / heads
    // batches of `heads` heads, the launch shape of the whole call.
    const int st = run_chunked(c, planes, a, 5, heads, [&](long long p0, long long p1, cudaStream_t s) {
        const long long off = p0 * seq * hd;
        return attention(reinterpret_cast<const float*>(a[0].dev) + off, reinterpret_cast<const float*>(a[1].dev) + off,
                         reinterpret_cast<const float*>(a[2].dev) + off, reinterpret_cast<const float*>(a[4].dev),
                         causal, reinterpret_cast<float*>(a[3].dev) + off, (int)((p1 - p0) / heads), heads, seq, hd, s);
    });
    return c.finish(st, false);
}
RAC_API void rac_attention(const float* q, const float* k, const float* v, const float* mask,
                           int is_causal, float* out, int batch, int n_heads, int seq, int head_dim) {
    set_status(do_attention(q, k, v, mask, is_causal, out, batch, n_heads, seq, head_dim), "rac_attention");
}

// ── context API (rac.h:85-88) ───────────────────────────────────────────

struct rac_context_t { rac_backend backend; int device; };

RAC_API rac_context rac_create_context(rac_backend backend) {
    if (backend != RAC_BACKEND_CUDA) { set_status(kErrUnsupported, "rac_create_context"); return nullptr; }
    int dev = 0;
    if (device_ready(&dev) != kOk) { set_status(kErrCuda, "rac_create_context"); return nullptr; }
    auto* ctx = static_cast<rac_context>(std::malloc(sizeof(rac_context_t)));
    if (!ctx) { set_status(kErrAlloc, "rac_create_context"); return nullptr; }
    ctx->backend = backend;
    ctx->device = dev;
    set_status(kOk, "rac_create_context");
    return ctx;
}
RAC_API void rac_destroy_context(rac_context ctx) { std::free(ctx); }

RAC_API int rac_query_capability(rac_context ctx, rac_op_type op) {
    (void)ctx;
    switch (op) {
        case RAC_OP_ROTATE: case RAC_OP_EXP: case RAC_OP_TANH: case RAC_OP_SOFTMAX:
        case RAC_OP_ROTATE_BATCH: case RAC_OP_MATMUL: case RAC_OP_RSQRT: case RAC_OP_SIGMOID:
        case RAC_OP_SINCOS: case RAC_OP_LAYERNORM: case RAC_OP_RMSNORM: case RAC_OP_ROPE_CACHE:
        case RAC_OP_ROPE_APPLY: case RAC_OP_ATTENTION:
            return 1;
        default:
            return 0;
    }
}

RAC_API int rac_execute(rac_context ctx, rac_op_type op, void* desc) {
    if (!ctx || !desc) return set_status(kErrNullPtr, "rac_execute");
    int prev = 0;
    cudaGetDevice(&prev);
    if (prev != ctx->device) cudaSetDevice(ctx->device);
    switch (op) {
        case RAC_OP_MATMUL: {
            auto* d = static_cast<rac_matmul_desc*>(desc);
            rac_matmul_ex(d->A, d->B, d->C, d->M, d->N, d->K, -1, -1);
            break;
        }
        case RAC_OP_ROTATE_BATCH: {
            auto* d = static_cast<rac_rotate_batch_desc*>(desc);
            if (d->iters <= 0) rac_rotate_batch(const_cast<float2*>(d->v), const_cast<float*>(d->theta), d->out, d->n);
            else rac_rotate_batch_n(d->v, d->theta, d->out, d->n, d->iters);
            break;
        }
        case RAC_OP_SOFTMAX: {
            auto* d = static_cast<rac_softmax_desc*>(desc);
            rac_softmax_batch(d->x, d->out, d->rows, d->n);
            break;
        }
        case RAC_OP_RMSNORM: {
            auto* d = static_cast<rac_norm_desc*>(desc);
            rac_rmsnorm(d->x, d->y, d->gamma, d->eps, d->rows, d->d);
            break;
        }
        case RAC_OP_LAYERNORM: {
            auto* d = static_cast<rac_norm_desc*>(desc);
            rac_layernorm(d->x, d->y, d->gamma, d->beta, d->eps, d->rows, d->d);
            break;
        }
        case RAC_OP_ROPE_APPLY: {
            auto* d = static_cast<rac_rope_apply_desc*>(desc);
            rac_rope_apply(d->x, d->cos_tab, d->sin_tab, d->batch, d->n_heads, d->seq, d->head_dim);
            break;
        }
        case RAC_OP_ROPE_CACHE: {
            auto* d = static_cast<rac_rope_cache_desc*>(desc);
            rac_rope_cache(d->cos_out, d->sin_out, d->max_seq, d->head_dim, d->base);
            break;
        }
        case RAC_OP_EXP: case RAC_OP_TANH: case RAC_OP_RSQRT: case RAC_OP_SIGMOID: {
            auto* d = static_cast<rac_unary_desc*>(desc);
            const int u = op == RAC_OP_EXP ? kUnaryExp : op == RAC_OP_TANH ? kUnaryTanh
                        : op == RAC_OP_RSQRT ? kUnaryRsqrt : kUnarySigmoid;
            set_status(do_unary(d->x, d->y, d->n, u), "rac_execute");
            break;
        }
        case RAC_OP_ATTENTION: {
            auto* d = static_cast<rac_attention_desc*>(desc);
            rac_attention(d->q, d->k, d->v, d->mask, d->is_causal, d->out, d->batch, d->n_heads,
                          d->seq, d->head_dim);
            break;
        }
        default:
            set_status(kErrUnsupported, "rac_execute");
    }
    const int st = t_status;
    if (prev != ctx->device) cudaSetDevice(prev);
    return st;
}
