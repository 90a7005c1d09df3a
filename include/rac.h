/*
 * rac.h -- RAC rotation-accumulate C API, served by librac_b200.so on B200.
 *
 * Host-callable subset of the reference interface (rac.h of
 * Pinnacle-Quantum-Group/RAC; each declaration cites the line it replaces).
 * Names, argument order and meaning are unchanged, so a caller of the
 * reference header relinks against librac_b200.so without source changes.
 *
 * Semantics of this implementation:
 *   - every computation runs on the current CUDA device (sm_100a kernels);
 *     there is no CPU fallback.  Without a usable GPU each call records
 *     RAC_ERR_CUDA in rac_last_error() (see rac_b200.h) and returns.
 *   - pointers may be host memory or device memory; host buffers are staged
 *     through device memory.  Calls are blocking, as C semantics require.
 *   - numerics follow the reference CPU library lib/c/rac_cpu.c.
 *
 * Declarations of the reference header that are outside the rotation-
 * accumulate hot path (rac_rotate_raw, rac_compensate, rac_project,
 * rac_polar, rac_norm, rac_normalize, rac_dot, rac_coherence,
 * rac_complex_mul, rac_dct, rac_inner, rac_outer) are not exported.
 * rac_attention (ref rac.h:330-335) is exported: the fused attention of the
 * RACLlamaBlock path.
 */
#ifndef RAC_H
#define RAC_H

#if defined(__CUDACC__)
  #include <cuda_runtime.h>
#else
  #if !defined(RAC_FLOAT2_DEFINED) && !defined(__VECTOR_TYPES_H__)
    #define RAC_FLOAT2_DEFINED
    typedef struct { float x; float y; } float2;   /* ref rac.h:31 */
  #endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define RAC_K_INV  0.60725f   /* ref rac.h:39 */
#define RAC_K      1.64676f   /* ref rac.h:40 */
#define RAC_ITERS  16         /* ref rac.h:41 */

/* ── context (ref rac.h:45-88) ──────────────────────────────────────────── */
typedef struct rac_context_t* rac_context;

typedef enum {
    RAC_BACKEND_CUDA = 0, RAC_BACKEND_HIP = 1, RAC_BACKEND_CPU = 2, RAC_BACKEND_FIL = 3
} rac_backend;

typedef enum {
    RAC_OP_ROTATE = 0, RAC_OP_ROTATE_RAW = 1, RAC_OP_PROJECT = 2, RAC_OP_POLAR = 3,
    RAC_OP_NORM = 4, RAC_OP_NORMALIZE = 5, RAC_OP_DOT = 6, RAC_OP_COHERENCE = 7,
    RAC_OP_COMPLEX_MUL = 8, RAC_OP_DCT = 9, RAC_OP_EXP = 10, RAC_OP_TANH = 11,
    RAC_OP_SOFTMAX = 12, RAC_OP_ROTATE_BATCH = 13, RAC_OP_INNER = 14, RAC_OP_OUTER = 15,
    RAC_OP_MATMUL = 16, RAC_OP_RSQRT = 17, RAC_OP_SIGMOID = 18, RAC_OP_SINCOS = 19,
    RAC_OP_LAYERNORM = 20, RAC_OP_RMSNORM = 21, RAC_OP_ROPE_CACHE = 22,
    RAC_OP_ROPE_APPLY = 23, RAC_OP_ATTENTION = 24, RAC_OP_EXTENDED = 0xFF
} rac_op_type;

/* ref rac.h:85.  Only RAC_BACKEND_CUDA yields a context (NULL otherwise). */
rac_context rac_create_context(rac_backend backend);
/* ref rac.h:86 */
void        rac_destroy_context(rac_context ctx);
/* ref rac.h:87.  1 for ops this library executes, 0 otherwise. */
int         rac_query_capability(rac_context ctx, rac_op_type op);
/* ref rac.h:88.  desc points to the rac_*_desc struct of rac_b200.h for op;
 * returns a rac_b200 status (0 = ok). */
int         rac_execute(rac_context ctx, rac_op_type op, void *desc);

/* ── 1. rotation (ref rac.h:101) ────────────────────────────────────────── */
float2 rac_rotate(float2 v, float theta);

/* ── 5. activations (ref rac.h:198, :205, :214) ─────────────────────────── */
float  rac_exp(float x);
float  rac_tanh(float x);
void   rac_softmax(float *x, float *out, int n);

/* ── 6. batch / linear algebra (ref rac.h:223, :249) ────────────────────── */
void   rac_rotate_batch(float2 *v, float *theta, float2 *out, int n);
/* C[M,N] = A[M,K] @ B[K,N], row-major.  Uses the process-wide mode and
 * iteration knobs (rac_b200.h: rac_set_cordic_mode/iters; defaults CORDIC,
 * RAC_ITERS). */
void   rac_matmul(float *A, float *B, float *C, int M, int N, int K);

/* ── 7. transformer primitives (ref rac.h:274-335) ──────────────────────── */
float  rac_rsqrt(float x);
float  rac_sigmoid(float x);
void   rac_sincos(float theta, float *s, float *c);
void   rac_layernorm(const float *x, float *y, const float *gamma,
                     const float *beta, float eps, int rows, int d);
void   rac_rmsnorm(const float *x, float *y, const float *gamma,
                   float eps, int rows, int d);
void   rac_rope_cache(float *cos_out, float *sin_out, int max_seq,
                      int head_dim, float base);
void   rac_rope_apply(float *x, const float *cos_tab, const float *sin_tab,
                      int batch, int n_heads, int seq, int head_dim);
/* ref rac.h:330-335.  q, k, v, out [batch, n_heads, seq, head_dim];
 * head_dim in {32, 64, 128}; mask optional [seq, seq] additive. */
void   rac_attention(const float *q, const float *k, const float *v,
                     const float *mask, int is_causal, float *out,
                     int batch, int n_heads, int seq, int head_dim);

/* ── 8. tunable precision (ref rac.h:345-346) ───────────────────────────── */
float2 rac_rotate_precision(float2 v, float theta, int iters);
float  rac_project_precision(float2 v, float theta, int iters);

#ifdef __cplusplus
}
#endif

#endif /* RAC_H */
