/*
 * rac_b200.h -- extensions of the RAC C API exported by librac_b200.so.
 *
 * Three groups:
 *  1. error channel and process-wide knobs (the reference binding keeps the
 *     same knobs in rac_torch/rac_torch_bind.cpp:54-55, :205-219);
 *  2. batch forms of the _n primitives of lib/c/rac_cpu.h:110-114 and the
 *     batch helpers of lib/c/rac_cpu.h (rac_softmax_batch);
 *  3. stream-ordered device entry points: the GEMM launchers of
 *     rac_torch/rac_kernels.hip:822-909 with the same names and argument
 *     meaning, plus *_async forms of every op for callers that own device
 *     memory and a cudaStream_t (passed as void*).  These never synchronise
 *     and return a status; the PyTorch layer binds to them.
 *
 * Status codes follow lib/c/rac_cpu.h:54-59 and extend them.
 */
#ifndef RAC_B200_H
#define RAC_B200_H

#include "rac.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ── 1. status, errors, knobs ───────────────────────────────────────────── */
#define RAC_OK               0
#define RAC_ERR_NULL_PTR    -1   /* lib/c/rac_cpu.h:56 */
#define RAC_ERR_INVALID_DIM -2   /* lib/c/rac_cpu.h:57 */
#define RAC_ERR_ALLOC       -3   /* lib/c/rac_cpu.h:58 */
#define RAC_ERR_CUDA        -4   /* no usable device, or a CUDA call failed */
#define RAC_ERR_UNSUPPORTED -5   /* op/mode/layout not provided */
#define RAC_ERR_DEVICE      -6   /* a kernel's bounded loop gave up (e.g. |theta| >= 2^25) */

#define RAC_MODE_FAST     0      /* rac_kernels.hip:13 */
#define RAC_MODE_CORDIC   1      /* rac_kernels.hip:14 */
#define RAC_MODE_SHIFTADD 2      /* rac_kernels.hip:15 (integer shift-add product) */

#define RAC_ACT_NONE 0           /* rac_torch.cu:665-666 activation ids */
#define RAC_ACT_RELU 1
#define RAC_ACT_GELU 2
#define RAC_ACT_SILU 3
/* Gated FFN (SwiGLU, bench/bench_rac_transformer.c:441-453) in one GEMM: B holds
 * the gate and up weights row-interleaved (gate row c at 2c, up row c at
 * 2c+1), and C gets N/2 columns, C[m, c] = silu(v[m, 2c]) * v[m, 2c+1] with
 * v = alpha * op(A) op(B) (+ bias).  N must be even and beta 0.  The same
 * bits as a SiLU GEMM over the gate rows times a plain GEMM over the up rows,
 * multiplied elementwise.  No counterpart in the reference's extension. */
#define RAC_ACT_SWIGLU 4

/* Thread-local status of the last call made on this thread (0 = ok). */
int         rac_last_error(void);
const char *rac_last_error_string(void);
void        rac_clear_error(void);

/* Process-wide GEMM knobs used by rac_matmul and by launchers given
 * iters <= 0 / mode < 0.  iters is clamped to [1, 24]; iters <= 0 resets to
 * the default.  Defaults: iters = RAC_ITERS (env RAC_CORDIC_ITERS),
  * mode = RAC_MODE_CORDIC (env RAC_CORDIC_MODE = fast|cordic|shiftadd). */
void rac_set_cordic_iters(int iters);
int  rac_get_cordic_iters(void);
void rac_set_cordic_mode(int mode);
int  rac_get_cordic_mode(void);

/* Library and device information. */
const char *rac_b200_version(void);
int  rac_b200_device_count(void);
/* The 24 direction signs d_i of the GEMM micro-rotation sequence (see
 * rac_torch/rac_kernels.hip:176-185); for tests. */
void rac_b200_cordic_gemm_directions(int out[24]);

/* ── 2. batch forms (host or device pointers, blocking) ─────────────────── */
/* out[i] = rac_rotate_n(v[i], theta[i], iters)  (lib/c/rac_cpu.c:275-280) */
void rac_rotate_batch_n(const float2 *v, const float *theta, float2 *out, int n, int iters);
/* out[i] = rac_project_n(v[i], theta[i], iters) (lib/c/rac_cpu.c:282-288) */
void rac_project_batch_n(const float2 *v, const float *theta, float *out, int n, int iters);
void rac_exp_batch(const float *x, float *y, int n);
void rac_tanh_batch(const float *x, float *y, int n);
void rac_rsqrt_batch(const float *x, float *y, int n);
void rac_sigmoid_batch(const float *x, float *y, int n);
void rac_sincos_batch(const float *theta, float *s, float *c, int n);
/* lib/c/rac_cpu.c:459-463 */
void rac_softmax_batch(const float *x, float *out, int batch, int n);
/* rac_matmul with explicit iteration count and mode (no knob). */
void rac_matmul_ex(const float *A, const float *B, float *C, int M, int N, int K,
                   int iters, int mode);

/* ── 3. stream-ordered device entry points ──────────────────────────────── */
/* rac_kernels.hip:822-909: C = alpha * op(A) op(B) + beta * C on `stream`
 * (a cudaStream_t), device pointers, row-major, contiguous.
 *   nn: A[M,K]  B[K,N];   nt: A[M,K]  B[N,K];   tn: A[K,M]  B[K,N].
 * iters <= 0 / mode < 0 take the process-wide knobs. */
void rac_launch_nn_iters(const float *A, const float *B, float *C, int M, int N, int K,
                         float alpha, float beta, int iters, int mode, void *stream);
void rac_launch_nt_iters(const float *A, const float *B, float *C, int M, int N, int K,
                         float alpha, float beta, int iters, int mode, void *stream);
void rac_launch_tn_iters(const float *A, const float *B, float *C, int M, int N, int K,
                         float alpha, float beta, int iters, int mode, void *stream);
/* rac_kernels.hip:886-909: FAST mode, the reference's legacy entry points. */
void rac_launch_nn(const float *A, const float *B, float *C, int M, int N, int K,
                   float alpha, float beta, void *stream);
void rac_launch_nt(const float *A, const float *B, float *C, int M, int N, int K,
                   float alpha, float beta, void *stream);
void rac_launch_tn(const float *A, const float *B, float *C, int M, int N, int K,
                   float alpha, float beta, void *stream);

/* General GEMM with strides and a fused epilogue:
 *   C = act(alpha * op(A) op(B) + beta * Cin + bias)
 * layout 0/1/2 = nn/nt/tn; Cin read only when beta != 0 (may equal C);
 * bias is [N] or NULL; act is RAC_ACT_*.  Covers rac_fused_linear_kernel
 * (rac_torch.cu:705-779) and residual-add fusion.  `variant` 0 = automatic
 * tile.  Returns a status. */
int rac_gemm_async(const float *A, long long lda, const float *B, long long ldb,
                   float *C, long long ldc, const float *Cin, long long ldcin,
                   const float *bias, int M, int N, int K, int layout, int mode,
                   int iters, float alpha, float beta, int act, int variant,
                   void *stream);

/* rac_gemm_async for callers that cannot allocate device memory -- no
 * counterpart in the reference.  Same arguments and result as
 * rac_gemm_async, always split-K (`splits` K chunks; 0 = the automatic
 * count, at least 1), with the partial sums held in a 16 MiB array compiled
 * into the library instead of a workspace allocated per call: the call makes
 * no allocation at all.  Hosts that give a library a fixed device-memory
 * budget, or cannot tolerate an allocation on a latency-critical path, use
 * this form.  Limits: splits * M * N <= 4 Mi floats (else
 * RAC_ERR_INVALID_DIM with the sizes in rac_last_error_string()); every GPU
 * that loads the library holds the 16 MiB until exit; all calls share the
 * array, so calls whose kernels overlap on the GPU (two streams, two host
 * threads) race.  The first call on a device looks the array's address up
 * (make it before any stream capture on that device). */
int rac_gemm_splitk_noalloc_async(const float *A, long long lda, const float *B, long long ldb,
                                  float *C, long long ldc, const float *Cin, long long ldcin,
                                  const float *bias, int M, int N, int K, int layout, int mode,
                                  int iters, float alpha, float beta, int act, int splits,
                                  void *stream);

int rac_rotate_batch_async(const float2 *v, const float *theta, float2 *out, long long n,
                           int iters, int literal_kinv, void *stream);
int rac_project_batch_async(const float2 *v, const float *theta, float *out, long long n,
                            int iters, void *stream);
int rac_sincos_batch_async(const float *theta, float *s, float *c, long long n, void *stream);
/* op: 0 exp, 1 tanh, 2 rsqrt, 3 sigmoid */
int rac_unary_async(const float *x, float *y, long long n, int op, void *stream);
int rac_softmax_async(const float *x, float *y, long long rows, int d, void *stream);
int rac_rmsnorm_async(const float *x, float *y, const float *gamma, float eps,
                      long long rows, int d, void *stream);
int rac_layernorm_async(const float *x, float *y, const float *gamma, const float *beta,
                        float eps, long long rows, int d, void *stream);
int rac_rope_cache_async(float *cos_out, float *sin_out, int max_seq, int head_dim,
                         float base, void *stream);
/* In place on [batch_heads, seq, head_dim]; pos (optional, device int32[seq])
 * maps sequence index -> table row.  form 0 = lib/c rac_rope_apply
 * (rac_cpu.c:600-635), form 1 = torch RACRoPE (rac_torch.py:1165-1181). */
int rac_rope_apply_async(float *x, const float *cos_tab, const float *sin_tab,
                         const int *pos, long long batch_heads, int seq, int head_dim,
                         int form, void *stream);
/* Fused attention on `stream` (device pointers): rac_attention without the
 * [seq, seq] score tensor (lib/c/rac_cpu.c:637-703 semantics). */
int rac_attention_async(const float *q, const float *k, const float *v, const float *mask,
                        int is_causal, float *out, int batch, int n_heads, int seq,
                        int head_dim, void *stream);
/* Reads and clears the device's error word (bounded-loop overruns) after
 * synchronising `stream`; returns RAC_OK or RAC_ERR_DEVICE. */
int rac_check_device_errors(void *stream);

/* ── op descriptors for rac_execute ─────────────────────────────────────── */
typedef struct { const float *A, *B; float *C; int M, N, K; } rac_matmul_desc;
typedef struct { const float2 *v; const float *theta; float2 *out; int n; int iters; } rac_rotate_batch_desc;
typedef struct { const float *x; float *out; int rows, n; } rac_softmax_desc;
typedef struct { const float *x; float *y; const float *gamma, *beta; float eps; int rows, d; } rac_norm_desc;
typedef struct { float *x; const float *cos_tab, *sin_tab; int batch, n_heads, seq, head_dim; } rac_rope_apply_desc;
typedef struct { float *cos_out, *sin_out; int max_seq, head_dim; float base; } rac_rope_cache_desc;
typedef struct { const float *x; float *y; int n; } rac_unary_desc;
typedef struct { const float *q, *k, *v, *mask; int is_causal; float *out;
                 int batch, n_heads, seq, head_dim; } rac_attention_desc;

#ifdef __cplusplus
}
#endif

#endif /* RAC_B200_H */
