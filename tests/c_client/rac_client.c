/* A C caller of the reference's rac.h API, linked against librac_b200.so.
 * Exercises rac_matmul, rac_rotate_batch, rac_rmsnorm, rac_softmax and the
 * context API with host buffers and checks the results against plain C
 * loops.  Exit code: 0 ok, 2 = no device (status RAC_ERR_CUDA reported),
 * 1 = wrong result. */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include "rac.h"
#include "rac_b200.h"

static float frand(unsigned *s) { *s = *s * 1664525u + 1013904223u; return (float)(*s >> 8) / 8388608.0f - 1.0f; }

int main(void) {
    enum { M = 70, N = 50, K = 90, NV = 1000, R = 4, D = 256 };
    static float A[M * K], B[K * N], C[M * N], theta[NV], x[R * D], y[R * D], g[D], sm[D];
    static float2 v[NV], out[NV];
    unsigned s = 12345u;
    for (int i = 0; i < M * K; i++) A[i] = frand(&s);
    for (int i = 0; i < K * N; i++) B[i] = frand(&s);
    for (int i = 0; i < NV; i++) { v[i].x = frand(&s); v[i].y = frand(&s); theta[i] = 3.0f * frand(&s); }
    for (int i = 0; i < R * D; i++) x[i] = frand(&s);
    for (int i = 0; i < D; i++) g[i] = 1.0f + 0.25f * frand(&s);

    rac_set_cordic_iters(16);
    rac_set_cordic_mode(RAC_MODE_CORDIC);
    rac_matmul(A, B, C, M, N, K);
    if (rac_last_error() == RAC_ERR_CUDA) { printf("no device: %s\n", rac_last_error_string()); return 2; }
    if (rac_last_error()) { printf("rac_matmul: %s\n", rac_last_error_string()); return 1; }
    double err = 0, ref_rms = 0;
    for (int i = 0; i < M; i++)
        for (int j = 0; j < N; j++) {
            double acc = 0;
            for (int k = 0; k < K; k++) acc += (double)A[i * K + k] * B[k * N + j];
            err = fmax(err, fabs(acc - C[i * N + j]));
            ref_rms += acc * acc;
        }
    ref_rms = sqrt(ref_rms / (M * N));
    if (err / ref_rms > 1e-4) { printf("matmul error %g\n", err / ref_rms); return 1; }

    rac_rotate_batch(v, theta, out, NV);
    for (int i = 0; i < NV; i++) {
        float c = cosf(theta[i]), sn = sinf(theta[i]);
        float ex = v[i].x * c - v[i].y * sn, ey = v[i].x * sn + v[i].y * c;
        if (fabsf(out[i].x - ex) > 1e-3f || fabsf(out[i].y - ey) > 1e-3f) { printf("rotate %d\n", i); return 1; }
    }
    rac_rmsnorm(x, y, g, 1e-6f, R, D);
    for (int r = 0; r < R; r++) {
        double ms = 0;
        for (int i = 0; i < D; i++) ms += (double)x[r * D + i] * x[r * D + i];
        double inv = 1.0 / sqrt(ms / D + 1e-6);
        for (int i = 0; i < D; i++)
            if (fabs(y[r * D + i] - x[r * D + i] * inv * g[i]) > 1e-5) { printf("rmsnorm\n"); return 1; }
    }
    rac_softmax(x, sm, D);
    double tot = 0;
    for (int i = 0; i < D; i++) tot += sm[i];
    if (fabs(tot - 1.0) > 1e-5) { printf("softmax sum %g\n", tot); return 1; }

    rac_context ctx = rac_create_context(RAC_BACKEND_CUDA);
    if (!ctx || !rac_query_capability(ctx, RAC_OP_MATMUL)) { printf("context\n"); return 1; }
    float C2[M * N];
    rac_matmul_desc md = {A, B, C2, M, N, K};
    if (rac_execute(ctx, RAC_OP_MATMUL, &md) != RAC_OK) { printf("execute\n"); return 1; }
    for (int i = 0; i < M * N; i++) if (C2[i] != C[i]) { printf("execute result\n"); return 1; }
    rac_destroy_context(ctx);
    printf("ok\n");
    return 0;
}
