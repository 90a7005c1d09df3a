// attention.cu -- fused scaled-dot-product attention (rac_attention), sm_100a.
//
// Semantics: lib/c/rac_cpu.c:637-703 (rac_scaled_dot_attention):
//   score[t,s] = fmaf-accumulated q_t . k_s (d ascending) * (1/sqrtf(hd)),
//   -inf where causal and s > t, + mask[t,s] when a mask is given,
//   p = expf(score - rowmax) / sum,  out_t = sum_s p[t,s] * v_s (s ascending).
//
// One CTA owns 64 query rows of one (batch, head) and streams the keys in
// 64-row tiles through shared memory; the [seq, seq] score matrix never
// exists in HBM.  Scores are accumulated over d in ascending order exactly as
// the reference does (bit-identical scores); the softmax is online -- a
// running row max with rescaling of the partial sum and of O -- and O
// accumulates e * V key by key in ascending order, scaled by 1/sum at the
// end.  The output differs from the reference by expf's last bit, the
// rescaling roundings and the sum's association (the reference multiplies by
// 1/sum before accumulating): within the reference's own distance from the
// exact result.  Deterministic (fixed tile order).
//
// 128 threads: for the 64x64 score tile a thread owns rows rg + 16i (i < 4) and
// columns cg + 8j (j < 8); for the 64 x HD output it owns the same rows and
// HD/8 columns in float4 groups.  Shared memory holds Q, K and V tiles
// (64 x HD each, unpadded) and the 64 x 64 P tile: 112 KB at HD = 128, so two
// CTAs fit on an SM.  Bank conflicts are avoided by layout, not padding:
//   * Q and K are stored with their float4 column XORed by (row & 7): the 8
//     K rows and the 4 Q rows a warp reads at one d fall in distinct 16-byte
//     bank groups;
//   * V reads are 8 consecutive float4 of one row;
//   * P is stored with its column XORed by (row & 3) << 3, so both the
//     scalar writes (4 rows x 8 columns per warp) and the reads (4 rows, one
//     column) hit distinct banks.
// The K and V tiles stream in with cp.async while the previous phase
// computes: V(kb) during the scores and softmax of tile kb, K(kb+1) during
// P V of tile kb.
#include <cmath>
#include <mutex>

#include "rac_internal.h"
#include "stream_ops.h"

namespace racb {

constexpr int kAttBQ = 64, kAttBK = 64, kAttThreads = 128;

template <int HD>
struct AttSmem {
    static_assert(HD % 32 == 0, "the K swizzle needs >= 8 float4 per row");
    static constexpr int PLD = kAttBK;
    static constexpr size_t bytes = sizeof(float) * (3 * kAttBQ * HD + kAttBQ * PLD);
};

// Float offset of element (row r, float4 column c4) of a swizzled Q or K tile.
template <int HD>
__device__ __forceinline__ int k_off(int r, int c4) { return r * HD + ((c4 ^ (r & 7)) << 2); }
// Float offset of element (row r, column c) of the swizzled P tile.
__device__ __forceinline__ int p_off(int r, int c) { return r * kAttBK + (c ^ ((r & 3) << 3)); }

// 16-byte asynchronous global->shared copy (cp.async.cg); a src size of 0
// zero-fills the destination (rows past the end of the sequence).
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
    const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;"
                 :: "r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Issues the copies of rows [row0, row0 + 64) of a [seq, HD] matrix into a
// tile (zeros past rows_valid) and commits them as one group.
template <int HD, bool SWZ>
__device__ __forceinline__ void load_tile_async(float* dst, const float* __restrict__ src, int row0,
                                                int rows_valid) {
    constexpr int QPR = HD / 4;                   // float4 per row
    for (int e = threadIdx.x; e < kAttBQ * QPR; e += kAttThreads) {
        const int r = e / QPR, c4 = e % QPR;
        const bool ok = row0 + r < rows_valid;
        const int o = SWZ ? k_off<HD>(r, c4) : r * HD + 4 * c4;
        cp_async16(dst + o, src + (long long)(ok ? row0 + r : 0) * HD + 4 * c4, ok);
    }
    cp_async_commit();
}

// Scores of this thread's 4 x 8 block for the key tile in Ks, after scale,
// causal and mask (keys beyond seq -> -inf).
template <int HD>
__device__ __forceinline__ void tile_scores(float (&sc)[4][8], const float* Qs, const float* Ks,
                                            int t0, int s0, int seq, float scale, int causal,
                                            const float* __restrict__ mask) {
    const int rg = threadIdx.x >> 3, cg = threadIdx.x & 7;
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) sc[i][j] = 0.0f;
#pragma unroll 4
    for (int d = 0; d < HD; d += 4) {
        float4 q[4], k[8];
        // K rows cg + 8j all have (row & 7) == cg, Q rows rg + 16i have
        // (row & 7) == (rg & 7): one swizzled column each for all j / i.
        const int kc = ((d >> 2) ^ cg) << 2;
        const int qc = ((d >> 2) ^ (rg & 7)) << 2;
#pragma unroll
        for (int i = 0; i < 4; ++i) q[i] = *reinterpret_cast<const float4*>(Qs + (rg + 16 * i) * HD + qc);
#pragma unroll
        for (int j = 0; j < 8; ++j) k[j] = *reinterpret_cast<const float4*>(Ks + (cg + 8 * j) * HD + kc);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float a = sc[i][j];
                a = __fmaf_rn(q[i].x, k[j].x, a);
                a = __fmaf_rn(q[i].y, k[j].y, a);
                a = __fmaf_rn(q[i].z, k[j].z, a);
                a = __fmaf_rn(q[i].w, k[j].w, a);
                sc[i][j] = a;
            }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + rg + 16 * i;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int s = s0 + cg + 8 * j;
            float v = __fmul_rn(sc[i][j], scale);
            if (causal && s > t) v = -INFINITY;
            if (mask && t < seq && s < seq) v = __fadd_rn(v, mask[(long long)t * seq + s]);
            if (s >= seq) v = -INFINITY;
            sc[i][j] = v;
        }
    }
}

template <int HD>
__global__ void __launch_bounds__(kAttThreads, 2)
k_attention(const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
            const float* __restrict__ mask, int causal, float* __restrict__ out, int heads, int seq,
            float scale) {
    constexpr int CG = HD / 32;
    extern __shared__ __align__(16) float smem[];
    float* Qs = smem;
    float* Ks = Qs + kAttBQ * HD;
    float* Vs = Ks + kAttBQ * HD;
    float* Ps = Vs + kAttBQ * HD;

    const int nqb = (seq + kAttBQ - 1) / kAttBQ;
    const int qb = nqb - 1 - blockIdx.x;          // heaviest (causal) blocks first
    const long long bh = (long long)blockIdx.z * heads + blockIdx.y;
    const float* qh = q + bh * seq * HD;
    const float* kh = k + bh * seq * HD;
    const float* vh = v + bh * seq * HD;
    float* oh = out + bh * seq * HD;
    const int t0 = qb * kAttBQ;
    const int rg = threadIdx.x >> 3, cg = threadIdx.x & 7;
    const int nkb = causal ? min(qb + 1, (seq + kAttBK - 1) / kAttBK) : (seq + kAttBK - 1) / kAttBK;

    load_tile_async<HD, true>(Qs, qh, t0, seq);
    load_tile_async<HD, true>(Ks, kh, 0, seq);

    // One pass with the running (online) row max m: per key tile,
    // m' = max(m, tile max), alpha = expf(m - m'), e = expf(s - m'),
    // l = l * alpha + sum e, O = O * alpha + e V (keys ascending).
    float mrow[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
    float lsum[4] = {0.f, 0.f, 0.f, 0.f};
    // O accumulators as packed pairs (columns 4c, 4c+1 and 4c+2, 4c+3): the
    // P V update is FFMA2, two FMAs per instruction, each rounded once.
    float2 o[4][CG][2];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int g = 0; g < CG; ++g) o[i][g][0] = o[i][g][1] = make_float2(0.f, 0.f);
    for (int kb = 0; kb < nkb; ++kb) {
        // V(kb) streams in during the scores and softmax of tile kb.
        load_tile_async<HD, false>(Vs, vh, kb * kAttBK, seq);
        cp_async_wait<1>();                       // Q and K(kb) have landed
        __syncthreads();
        float sc[4][8];
        tile_scores<HD>(sc, Qs, Ks, t0, kb * kAttBK, seq, scale, causal, mask);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float tm = sc[i][0];
#pragma unroll
            for (int j = 1; j < 8; ++j) tm = fmaxf(tm, sc[i][j]);
#pragma unroll
            for (int off = 1; off < 8; off <<= 1) tm = fmaxf(tm, __shfl_xor_sync(0xffffffffu, tm, off));
            const float mn = fmaxf(mrow[i], tm);
            // Rows with no finite score yet contribute nothing (their e = 0).
            const float alpha = (mn == -INFINITY) ? 1.0f : expf(__fsub_rn(mrow[i], mn));
            mrow[i] = mn;
            lsum[i] = __fmul_rn(lsum[i], alpha);
            const float2 a2 = make_float2(alpha, alpha);
#pragma unroll
            for (int g = 0; g < CG; ++g) {
                o[i][g][0] = __fmul2_rn(o[i][g][0], a2);
                o[i][g][1] = __fmul2_rn(o[i][g][1], a2);
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float e = (mn == -INFINITY) ? 0.0f : expf(__fsub_rn(sc[i][j], mn));
                lsum[i] = __fadd_rn(lsum[i], e);
                Ps[p_off(rg + 16 * i, cg + 8 * j)] = e;
            }
        }
        __syncthreads();                          // P visible, K(kb) no longer read
        // K(kb+1) streams in during P V of tile kb.
        if (kb + 1 < nkb) {
            load_tile_async<HD, true>(Ks, kh, (kb + 1) * kAttBK, seq);
            cp_async_wait<1>();                   // V(kb) has landed
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int kmax = min(kAttBK, seq - kb * kAttBK);
        auto pv_key = [&](int s, const float (&p)[4]) {
            float2 pd[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) pd[i] = make_float2(p[i], p[i]);
#pragma unroll
            for (int g = 0; g < CG; ++g) {
                const float4 vv = *reinterpret_cast<const float4*>(Vs + s * HD + cg * 4 + 32 * g);
                const float2 v01 = make_float2(vv.x, vv.y), v23 = make_float2(vv.z, vv.w);
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    o[i][g][0] = __ffma2_rn(pd[i], v01, o[i][g][0]);
                    o[i][g][1] = __ffma2_rn(pd[i], v23, o[i][g][1]);
                }
            }
        };
        int s = 0;
        // Four keys per P read: columns s..s+3 stay adjacent under the P
        // swizzle (it flips bits 3-4 of the column), so one float4 per row.
        for (; s + 4 <= kmax; s += 4) {
            float4 p4[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) p4[i] = *reinterpret_cast<const float4*>(Ps + p_off(rg + 16 * i, s));
            { const float p[4] = {p4[0].x, p4[1].x, p4[2].x, p4[3].x}; pv_key(s, p); }
            { const float p[4] = {p4[0].y, p4[1].y, p4[2].y, p4[3].y}; pv_key(s + 1, p); }
            { const float p[4] = {p4[0].z, p4[1].z, p4[2].z, p4[3].z}; pv_key(s + 2, p); }
            { const float p[4] = {p4[0].w, p4[1].w, p4[2].w, p4[3].w}; pv_key(s + 3, p); }
        }
        for (; s < kmax; ++s) {
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = Ps[p_off(rg + 16 * i, s)];
            pv_key(s, p);
        }
        __syncthreads();                          // V and P free for the next tile
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int off = 1; off < 8; off <<= 1) lsum[i] = __fadd_rn(lsum[i], __shfl_xor_sync(0xffffffffu, lsum[i], off));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int t = t0 + rg + 16 * i;
        if (t >= seq) continue;
        // A row whose scores are all -inf gives NaN, as in the reference
        // (expf(-inf - -inf) there); otherwise inv = 1/sum (sum > 0).
        const float inv = mrow[i] == -INFINITY ? __int_as_float(0x7fc00000)
                        : (lsum[i] > 0.0f ? __fdiv_rn(1.0f, lsum[i]) : 0.0f);
#pragma unroll
        for (int g = 0; g < CG; ++g) {
            const float2 r0 = o[i][g][0], r1 = o[i][g][1];
            *reinterpret_cast<float4*>(oh + (long long)t * HD + cg * 4 + 32 * g) =
                make_float4(__fmul_rn(r0.x, inv), __fmul_rn(r0.y, inv), __fmul_rn(r1.x, inv), __fmul_rn(r1.y, inv));
        }
    }
}

template <int HD>
static int launch_att(const float* q, const float* k, const float* v, const float* mask, int causal,
                      float* out, int batch, int heads, int seq, float scale, cudaStream_t s) {
    const size_t smem = AttSmem<HD>::bytes;
    static std::once_flag once[64];
    static cudaError_t attr_err[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return kErrUnsupported;
    std::call_once(once[dev], [dev, smem] {
        attr_err[dev] = cudaFuncSetAttribute(k_attention<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (attr_err[dev] != cudaSuccess) return kErrCuda;
    const dim3 grid((seq + kAttBQ - 1) / kAttBQ, heads, batch);
    if (grid.y > 65535 || grid.z > 65535) return kErrInvalidDim;
    k_attention<HD><<<grid, kAttThreads, smem, s>>>(q, k, v, mask, causal, out, heads, seq, scale);
    return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int attention(const float* q, const float* k, const float* v, const float* mask, int causal,
              float* out, int batch, int heads, int seq, int head_dim, cudaStream_t s) {
    if (!q || !k || !v || !out) return kErrNullPtr;
    if (batch <= 0 || heads <= 0 || seq <= 0 || head_dim <= 0) return kErrInvalidDim;
    for (const void* p : {(const void*)q, (const void*)k, (const void*)v, (const void*)out})
        if (reinterpret_cast<uintptr_t>(p) & 15u) return kErrUnsupported;
    const float scale = 1.0f / sqrtf((float)head_dim);   // rac_cpu.c:646
    switch (head_dim) {
        case 32: return launch_att<32>(q, k, v, mask, causal, out, batch, heads, seq, scale, s);
        case 64: return launch_att<64>(q, k, v, mask, causal, out, batch, heads, seq, scale, s);
        case 128: return launch_att<128>(q, k, v, mask, causal, out, batch, heads, seq, scale, s);
        default: return kErrUnsupported;
    }
}

}  // namespace racb
