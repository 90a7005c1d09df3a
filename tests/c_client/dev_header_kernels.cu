// Test kernels for include/rac_b200_device.cuh: one element (or one dot
// product) per thread, results compared with the library's batch entry
// points by tests/test_device_header.py.
#include "rac_b200_device.cuh"

__global__ void k_elementwise(const float2* v, const float* th, int n, int iters, float2* rot,
                              float2* rotn, float* proj, float* s, float* c) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    rot[i] = rac_dev_rotate(v[i], th[i]);
    rotn[i] = rac_dev_rotate_n(v[i], th[i], iters);
    proj[i] = rac_dev_project_n(v[i], th[i], iters);
    rac_dev_sincos(th[i], &s[i], &c[i]);
}

// out[i] = sum_k A[i, k] * b[k] by chained CORDIC MACs (k ascending).
__global__ void k_dot(const float* A, const float* b, int n, int K, int iters, float* out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float acc = 0.0f;
    for (int k = 0; k < K; ++k) acc = rac_dev_fma_cordic(acc, A[(long long)i * K + k], b[k], iters);
    out[i] = acc;
}

extern "C" int run_elementwise(const float2* v, const float* th, int n, int iters, float2* rot,
                               float2* rotn, float* proj, float* s, float* c) {
    k_elementwise<<<(n + 127) / 128, 128>>>(v, th, n, iters, rot, rotn, proj, s, c);
    return (int)cudaDeviceSynchronize();
}

extern "C" int run_dot(const float* A, const float* b, int n, int K, int iters, float* out) {
    k_dot<<<(n + 127) / 128, 128>>>(A, b, n, K, iters, out);
    return (int)cudaDeviceSynchronize();
}
