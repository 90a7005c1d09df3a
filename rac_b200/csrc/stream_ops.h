// stream_ops.h -- internal launchers of the elementwise and row-wise kernels.
// All take device pointers, enqueue on `s`, never synchronise, and return a
// racb::Status.
#pragma once
#include <cuda_runtime.h>

namespace racb {

enum UnaryOp : int { kUnaryExp = 0, kUnaryTanh = 1, kUnaryRsqrt = 2, kUnarySigmoid = 3 };

int rotate_batch(const float2* v, const float* th, float2* out, long long n, int iters,
                 int literal_kinv, cudaStream_t s);
int project_batch(const float2* v, const float* th, float* out, long long n, int iters,
                  cudaStream_t s);
int sincos_batch(const float* th, float* s_out, float* c_out, long long n, cudaStream_t s);
int unary_batch(const float* x, float* y, long long n, int op, cudaStream_t s);
int rope_cache(float* cos_out, float* sin_out, int max_seq, int head_dim, float base,
               cudaStream_t s);
int rope_apply(float* x, const float* cos_tab, const float* sin_tab, const int* pos,
               long long batch_heads, int seq, int head_dim, int form, cudaStream_t s);

// Row-wise (rows x d, row-major, leading dimension d).
int softmax_rows(const float* x, float* y, long long rows, int d, cudaStream_t s);
int rmsnorm_rows(const float* x, float* y, const float* gamma, float eps, long long rows,
                 int d, cudaStream_t s);
int layernorm_rows(const float* x, float* y, const float* gamma, const float* beta, float eps,
                   long long rows, int d, cudaStream_t s);

// Fused attention (attention.cu), q/k/v/out [batch, heads, seq, head_dim]
// contiguous; mask optional [seq, seq]; head_dim in {32, 64, 128}.
int attention(const float* q, const float* k, const float* v, const float* mask, int causal,
              float* out, int batch, int heads, int seq, int head_dim, cudaStream_t s);

}  // namespace racb
