// gemm_dispatch.cu -- picks the GEMM kernel instance for a call.
#include "gemm_kernel.cuh"

namespace racb {

#define E4(MODE, ITERS, LAY) RACB_GEMM_EXTERN(MODE, ITERS, LAY, 1, true) \
    RACB_GEMM_EXTERN(MODE, ITERS, LAY, 1, false) RACB_GEMM_EXTERN(MODE, ITERS, LAY, 3, true) \
    RACB_GEMM_EXTERN(MODE, ITERS, LAY, 3, false)
E4(kFast, 0, kNN) E4(kFast, 0, kNT) E4(kFast, 0, kTN)
E4(kCordic, 0, kNN) E4(kCordic, 0, kNT) E4(kCordic, 0, kTN)
#define E2(ITERS) RACB_GEMM_EXTERN(kCordic, ITERS, kNN, 1, true) \
    RACB_GEMM_EXTERN(kCordic, ITERS, kNT, 1, true) RACB_GEMM_EXTERN(kCordic, ITERS, kNN, 3, true) \
    RACB_GEMM_EXTERN(kCordic, ITERS, kNT, 3, true)
E2(8) E2(16) E2(24)

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
    if (layout == kNN) return pick_tile<kCordic, ITERS, kNN>(p, v, true, s);
    return pick_tile<kCordic, ITERS, kNT>(p, v, true, s);
}

static bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

int launch_gemm(const GemmParams& p_in, int layout, int mode, int variant, cudaStream_t s) {
    if (p_in.M <= 0 || p_in.N <= 0 || p_in.K <= 0) return kErrInvalidDim;
    if (!p_in.A || !p_in.B || !p_in.C) return kErrNullPtr;
    if (layout < kNN || layout > kTN) return kErrUnsupported;
    if (p_in.beta != 0.0f && !p_in.Cin) return kErrNullPtr;
    GemmParams p = p_in;
    const int v = (variant == 1 || variant == 3) ? variant : (p.M <= 32 ? 3 : 1);
    // Vector loads need 16-byte aligned bases, leading dims that are
    // multiples of 4 and contiguous extents that are multiples of 4.
    const int a_contig = (layout == kTN) ? p.M : p.K;
    const int b_contig = (layout == kNT) ? p.K : p.N;
    const bool vec = aligned16(p.A) && aligned16(p.B) && (p.lda % 4 == 0) &&
                     (p.ldb % 4 == 0) && (a_contig % 4 == 0) && (b_contig % 4 == 0);
    if (mode == kFast) return pick_layout<kFast, 0>(p, layout, v, vec, s);
    if (mode != kCordic) return kErrUnsupported;
    if (p.iters < 1 || p.iters > kMaxIters) return kErrInvalidDim;
    p.k_inv = k_inv_of(p.iters);
    for (int i = 0; i < 24; ++i) p.coef[i] = gemm_coef(i);
    const bool fixed = vec && layout != kTN;
    if (fixed && p.iters == 8) return pick_fixed<8>(p, layout, v, s);
    if (fixed && p.iters == 16) return pick_fixed<16>(p, layout, v, s);
    if (fixed && p.iters == 24) return pick_fixed<24>(p, layout, v, s);
    return pick_layout<kCordic, 0>(p, layout, v, vec, s);
}

}  // namespace racb
