// gemm_dispatch.cu -- picks the GEMM kernel instance for a call.
#include <atomic>
#include <cstdlib>
#include <cudaTypedefs.h>
#include <mutex>

#include "gemm_fast.cuh"

namespace racb {

RACB_FAST_TMA_EXTERN(kNN, 1) RACB_FAST_TMA_EXTERN(kTN, 1) RACB_FAST_TMA_EXTERN(kNN, 2) RACB_FAST_TMA_EXTERN(kTN, 2)

// FAST mode on operands that meet the TMA rules and no split-K: the
// TMA-staged FFMA2 kernels (gemm_fast.cuh) -- NN / TN with 64 x 128 x 32 tiles (or
// 128 x 128 when variant bit 0x2000 asks), NT with swizzled k-major tiles
// (not with the SwiGLU epilogue).  Everything else (unaligned operands,
// split-K, variant bit 0x400) runs the general kernel.
static int pick_fast_tma(const GemmParams& p, int layout, int variant, cudaStream_t s) {
    if (p.ws || (variant & 0x400)) return kErrUnsupported;
    if (layout == kNT) return launch_fast_tma_nt(p, s);
    if (variant & 0x2000)
        return layout == kNN ? launch_fast_tma<kNN, 1>(p, s) : launch_fast_tma<kTN, 1>(p, s);

    return layout == kNN ? launch_fast_tma<kNN, 2>(p, s) : launch_fast_tma<kTN, 2>(p, s);
}

#define E4(MODE, ITERS, LAY) RACB_GEMM_EXTERN(MODE, ITERS, LAY, 1, true) \
    RACB_GEMM_EXTERN(MODE, ITERS, LAY, 1, false) RACB_GEMM_EXTERN(MODE, ITERS, LAY, 3, true) \
    RACB_GEMM_EXTERN(MODE, ITERS, LAY, 3, false)
E4(kFast, 0, kNN) E4(kFast, 0, kNT) E4(kFast, 0, kTN)
E4(kCordic, 0, kNN) E4(kCordic, 0, kNT) E4(kCordic, 0, kTN)
E4(kShiftAdd, 0, kNN) E4(kShiftAdd, 0, kNT) E4(kShiftAdd, 0, kTN)
#define E2(ITERS) RACB_GEMM_EXTERN(kCordic, ITERS, kNN, 1, true) \
    RACB_GEMM_EXTERN(kCordic, ITERS, kNT, 1, true) RACB_GEMM_EXTERN(kCordic, ITERS, kNN, 3, true) \
    RACB_GEMM_EXTERN(kCordic, ITERS, kNT, 3, true) RACB_GEMM_EXTERN(kCordic, ITERS, kNN, 2, true) \
    RACB_GEMM_EXTERN(kCordic, ITERS, kNT, 2, true) RACB_GEMM_EXTERN(kCordic, ITERS, kNN, 4, true) \
    RACB_GEMM_EXTERN(kCordic, ITERS, kNT, 4, true)
E2(8) E2(16) E2(24)
#define ET(ITERS) RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNN, 1) RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNT, 1) \
    RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNN, 2) RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNT, 2) \
    RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNN, 3) RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNT, 3) \
    RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNN, 4) RACB_GEMM_EXTERN_TMA(kCordic, ITERS, kNT, 4)
ET(8) ET(16) ET(24)

template <int ITERS, int LAYOUT>
static int launch_tma_tile(const GemmParams& p, int v, cudaStream_t s) {
    switch (v) {
        case 2: return launch_inst<kCordic, ITERS, LAYOUT, 2, true, true>(p, s);
        case 3: return launch_inst<kCordic, ITERS, LAYOUT, 3, true, true>(p, s);
        case 4: return launch_inst<kCordic, ITERS, LAYOUT, 4, true, true>(p, s);
        default: return launch_inst<kCordic, ITERS, LAYOUT, 1, true, true>(p, s);
    }
}

template <int ITERS>
static int pick_fixed_tma(const GemmParams& p, int layout, int v, cudaStream_t s) {
    return layout == kNN ? launch_tma_tile<ITERS, kNN>(p, v, s) : launch_tma_tile<ITERS, kNT>(p, v, s);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
        cudaGetLastError();
    });
    return fn;
}

bool encode_tensor_2d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer,
                      long long ld, uint32_t box_inner, uint32_t box_outer, bool swizzle128) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    if ((reinterpret_cast<uintptr_t>(base) & 15u) || ((ld * 4) & 15)) return false;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * sizeof(float)};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box,
               estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_2d(CUtensorMap* map, const float* base, uint64_t inner, uint64_t outer,
                      long long ld, uint32_t box_inner, uint32_t box_outer) {
    return encode_tensor_2d(map, base, inner, outer, ld, box_inner, box_outer, false);
}

bool make_tensor_maps(GemmParams& p, int layout, int BM, int BN, int BK) {
    // Boxes start at k multiples of BK and m / n multiples of BM / BN, so the
    // innermost coordinate of every copy is a multiple of 8 floats (32 B).
    const bool a_ok = layout == kTN ? encode_2d(&p.tmA, p.A, p.M, p.K, p.lda, BM, BK)
                                    : encode_2d(&p.tmA, p.A, p.K, p.M, p.lda, BK, BM);
    const bool b_ok = layout == kNT ? encode_2d(&p.tmB, p.B, p.K, p.N, p.ldb, BK, BN)
                                    : encode_2d(&p.tmB, p.B, p.N, p.K, p.ldb, BN, BK);
    return a_ok && b_ok;
}

// TMA staging for the fixed-n CORDIC kernels: variant bit 0x100 forces it,
// 0x200 forces the register-staged loader, otherwise env RAC_GEMM_TMA (1/0).
static bool use_tma(int variant) {
    if (variant & 0x100) return true;
    if (variant & 0x200) return false;
    static const bool env = [] {
        const char* e = std::getenv("RAC_GEMM_TMA");
        return !(e && e[0] == '0');
    }();
    return env;
}

template <int MODE, int ITERS, int LAYOUT>
static int pick_tile(const GemmParams& p, int v, bool vec, cudaStream_t s) {
    if (v == 3) return vec ? launch_inst<MODE, ITERS, LAYOUT, 3, true>(p, s)
                           : launch_inst<MODE, ITERS, LAYOUT, 3, false>(p, s);
    return vec ? launch_inst<MODE, ITERS, LAYOUT, 1, true>(p, s)
               : launch_inst<MODE, ITERS, LAYOUT, 1, false>(p, s);
}

template <int MODE, int ITERS>
static int pick_layout(const GemmParams& p, int layout, int v, bool vec, cudaStream_t s) {
    switch (layout) {
        case kNN: return pick_tile<MODE, ITERS, kNN>(p, v, vec, s);
        case kNT: return pick_tile<MODE, ITERS, kNT>(p, v, vec, s);
        case kTN: return pick_tile<MODE, ITERS, kTN>(p, v, vec, s);
        default: return kErrUnsupported;
    }
}

template <int ITERS>
static int pick_fixed(const GemmParams& p, int layout, int v, cudaStream_t s) {
    if (v == 2) return layout == kNN ? launch_inst<kCordic, ITERS, kNN, 2, true>(p, s)
                                     : launch_inst<kCordic, ITERS, kNT, 2, true>(p, s);
    if (v == 4) return layout == kNN ? launch_inst<kCordic, ITERS, kNN, 4, true>(p, s)
                                     : launch_inst<kCordic, ITERS, kNT, 4, true>(p, s);
    if (layout == kNN) return pick_tile<kCordic, ITERS, kNN>(p, v, true, s);
    return pick_tile<kCordic, ITERS, kNT>(p, v, true, s);
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static int sm_count() {
    static std::atomic<int> cached[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (!n) {
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

void keep_device_pool() {
    static std::once_flag once[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) { cudaGetLastError(); return; }
    std::call_once(once[dev], [dev] {
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
            unsigned long long thr = ~0ull;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
        }
        cudaGetLastError();
    });
}

static int sm_count();

// 3 for M <= 32.  Otherwise the 64x64 or 32x64 tile that minimises the work
// of the most loaded SM, ceil(tiles / SMs) x tile area -- the GEMM is
// issue-bound per SM, so that is its run time; ties go to the larger tile.
// The 64x128 tile (8x8 per thread) is not chosen automatically: its unrolled
// k-step is twice as long, and at n = 16 / 24 it measured 2 % / 28 % slower
// than 64x64 (instruction-cache pressure).  Kernels without the 64x64 and
// 32x64 instances (FAST, SHIFTADD, run-time n) use 64x128.  Variants 1-4 can
// be forced.
static int tile_variant(const GemmParams& p, int variant) {
    if (variant >= 1 && variant <= 4) return variant;
    if (p.M <= 32) return 3;
    const long long sms = sm_count();
    const int bms[2] = {64, 32}, bns[2] = {64, 64}, vs[2] = {2, 4};
    int best = 2;
    long long best_cost = -1;
    for (int i = 0; i < 2; ++i) {
        const long long tiles = (long long)((p.M + bms[i] - 1) / bms[i]) * ((p.N + bns[i] - 1) / bns[i]);
        const long long cost = (tiles + sms - 1) / sms * bms[i] * bns[i];
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = vs[i]; }
    }
    return best;
}

// Split-K when the output tiles cannot fill the machine: fewer tiles than
// SMs and K >= 1024.  S is chosen to minimise the most loaded SM's share of
// the work, ceil(tiles * S / SMs) / S, over 2 <= S <= K / 256 (chunks keep at
// least 256 k-steps); ties go to the smaller S.  variant 10+S forces S splits.
int splitk_count(const GemmParams& p, int layout, int mode, int variant) {
    (void)layout; (void)mode;
    const int v = tile_variant(p, variant);
    const int bm = v == 3 ? TileCfg<3>::BM : v == 4 ? TileCfg<4>::BM : TileCfg<1>::BM;
    const int bn = v == 3 ? TileCfg<3>::BN : (v == 2 || v == 4) ? 64 : TileCfg<1>::BN;
    const long long tiles = (long long)((p.M + bm - 1) / bm) * ((p.N + bn - 1) / bn);
    int S = 1;
    if (variant >= 10) {
        S = variant - 10;
    } else if (variant == 0 && tiles < sm_count() && p.K >= 1024) {
        const long long sms = sm_count();
        double best = 1.0;                                   // S = 1: the whole tile on one SM
        for (int c = 2; c <= p.K / 256; ++c) {
            const double share = (double)((tiles * c + sms - 1) / sms) / c;
            if (share < best - 1e-9) { best = share; S = c; }
        }
    }
    if (S < 1) S = 1;
    if (S > p.K) S = p.K;
    return S;
}

__global__ void __launch_bounds__(256) k_splitk_reduce(const GemmParams p) {
    const long long mn = (long long)p.M * p.N;
    if (p.act == kActSwiGLU) {                  // one output per (gate, up) column pair
        const int nh = p.N >> 1;
        for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < mn / 2;
             e += (long long)gridDim.x * blockDim.x) {
            const int gm = (int)(e / nh), c = (int)(e % nh);
            const long long e0 = (long long)gm * p.N + 2 * c;
            float g = p.ws[e0], u = p.ws[e0 + 1];
            for (int z = 1; z < p.splits; ++z) {
                g = __fadd_rn(g, p.ws[z * mn + e0]);
                u = __fadd_rn(u, p.ws[z * mn + e0 + 1]);
            }
            g = __fmul_rn(p.alpha, g);
            u = __fmul_rn(p.alpha, u);
            if (p.bias) { g = __fadd_rn(g, p.bias[2 * c]); u = __fadd_rn(u, p.bias[2 * c + 1]); }
            p.C[(long long)gm * p.ldc + c] = __fmul_rn(apply_act(g, kActSilu), u);
        }
        return;
    }
    for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < mn;
         e += (long long)gridDim.x * blockDim.x) {
        float acc = p.ws[e];
        for (int z = 1; z < p.splits; ++z) acc = __fadd_rn(acc, p.ws[z * mn + e]);
        const int gm = (int)(e / p.N), gn = (int)(e % p.N);
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

int launch_splitk_reduce(const GemmParams& p, cudaStream_t s) {
    const long long mn = (long long)p.M * p.N;
    long long blocks = (mn + 255) / 256;
    const long long cap = 8LL * sm_count();
    if (blocks > cap) blocks = cap;
    k_splitk_reduce<<<(int)blocks, 256, 0, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}


int launch_gemm(const GemmParams& p_in, int layout, int mode, int variant, cudaStream_t s) {
    if (p_in.M <= 0 || p_in.N <= 0 || p_in.K <= 0) return kErrInvalidDim;
    if (!p_in.A || !p_in.B || !p_in.C) return kErrNullPtr;
    if (layout < kNN || layout > kTN) return kErrUnsupported;
    if (p_in.beta != 0.0f && !p_in.Cin) return kErrNullPtr;
    if (p_in.act == kActSwiGLU && ((p_in.N & 1) || p_in.beta != 0.0f)) return kErrUnsupported;
    const int S = splitk_count(p_in, layout, mode, variant & 0xff);
    if (S <= 1) {
        GemmParams p = p_in;
        p.ws = nullptr; p.splits = 1; p.kchunk = 0;
        return launch_gemm_into(p, layout, mode, variant, s);
    }
    // Workspace from the device's stream-ordered pool (cached across calls).
    keep_device_pool();
    GemmParams p = p_in;
    p.kchunk = ((p.K + S - 1) / S + 7) / 8 * 8;             // multiple of BK
    p.splits = (p.K + p.kchunk - 1) / p.kchunk;
    const size_t bytes = sizeof(float) * (size_t)p.splits * p.M * p.N;
    if (cudaMallocAsync(reinterpret_cast<void**>(&p.ws), bytes, s) != cudaSuccess) {
        cudaGetLastError();
        return kErrAlloc;
    }
    int st = launch_gemm_into(p, layout, mode, variant, s);
    if (st == kOk) st = launch_splitk_reduce(p, s);
    cudaFreeAsync(p.ws, s);
    return st;
}

// Launches the tile kernel for p as given (p.ws / p.splits / p.kchunk set by
// the caller: ws == nullptr means no split).
int launch_gemm_into(const GemmParams& p_in, int layout, int mode, int variant, cudaStream_t s) {
    GemmParams p = p_in;
    const bool tma = use_tma(variant);
    const int hooks = variant;
    variant &= 0xff;
    int v = tile_variant(p, variant);
    int dev = 0;
    cudaGetDevice(&dev);
    p.err = device_error_word(dev);
    // Variant bit 0x1000 is a test hook: each stage barrier expects 16 bytes
    // more than its copies deliver and gives up after 4096 polls, so the
    // bounded-wait path (error word bit 1, no hang) can be exercised.
    p.tma_wait_limit = (hooks & 0x1000) ? 4096u : kTmaWaitLimit;
    p.tma_extra_tx = (hooks & 0x1000) ? 16u : 0u;
    // Vector loads need 16-byte aligned bases, leading dims that are
    // multiples of 4 and contiguous extents that are multiples of 4.
    const int a_contig = (layout == kTN) ? p.M : p.K;
    const int b_contig = (layout == kNT) ? p.K : p.N;
    const bool vec = aligned16(p.A) && aligned16(p.B) && (p.lda % 4 == 0) &&
                     (p.ldb % 4 == 0) && (a_contig % 4 == 0) && (b_contig % 4 == 0);
    if (mode == kFast) {
        if (vec && v != 3) {
            const int st = pick_fast_tma(p, layout, hooks, s);
            if (st != kErrUnsupported) return st;
        }
        return pick_layout<kFast, 0>(p, layout, (v == 2 || v == 4) ? 1 : v, vec, s);
    }
    if (mode == kShiftAdd) {
        if (p.iters < 1 || p.iters > kMaxIters) return kErrInvalidDim;
        return pick_layout<kShiftAdd, 0>(p, layout, (v == 2 || v == 4) ? 1 : v, vec, s);
    }
    if (mode != kCordic) return kErrUnsupported;
    if (p.iters < 1 || p.iters > kMaxIters) return kErrInvalidDim;
    p.k_inv = k_inv_of(p.iters);
    for (int i = 0; i < 24; ++i) p.coef[i] = gemm_coef(i);
    const bool fixed = vec && layout != kTN && (p.iters == 8 || p.iters == 16 || p.iters == 24);
    if ((v == 2 || v == 4) && !fixed) v = 1;   // tiles 2 and 4 exist for the fixed-n kernels only
    if (fixed && tma) {
        GemmParams q = p;
        if (make_tensor_maps(q, layout, 64, 64, 8)) {        // operands meet the TMA rules
            if (p.iters == 8) return pick_fixed_tma<8>(p, layout, v, s);
            if (p.iters == 16) return pick_fixed_tma<16>(p, layout, v, s);
            return pick_fixed_tma<24>(p, layout, v, s);
        }
    }
    if (fixed && p.iters == 8) return pick_fixed<8>(p, layout, v, s);
    if (fixed && p.iters == 16) return pick_fixed<16>(p, layout, v, s);
    if (fixed && p.iters == 24) return pick_fixed<24>(p, layout, v, s);
    return pick_layout<kCordic, 0>(p, layout, v, vec, s);
}

}  // namespace racb
