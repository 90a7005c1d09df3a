// CORDIC GEMM, n = 16 iterations unrolled: NN and NT layouts, vector loads, tiles 1-4.
#include "gemm_kernel.cuh"
namespace racb {
RACB_GEMM_INST(kCordic, 16, kNN, 1, true) RACB_GEMM_INST(kCordic, 16, kNT, 1, true)
RACB_GEMM_INST(kCordic, 16, kNN, 3, true) RACB_GEMM_INST(kCordic, 16, kNT, 3, true)
RACB_GEMM_INST(kCordic, 16, kNN, 2, true) RACB_GEMM_INST(kCordic, 16, kNT, 2, true)
RACB_GEMM_INST(kCordic, 16, kNN, 4, true) RACB_GEMM_INST(kCordic, 16, kNT, 4, true)
}
