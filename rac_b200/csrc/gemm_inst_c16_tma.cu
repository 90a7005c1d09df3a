// CORDIC GEMM, n = 16 iterations unrolled, TMA-staged: NN and NT, tiles 1-4.
#include "gemm_kernel.cuh"
namespace racb {
RACB_GEMM_INST_TMA(kCordic, 16, kNN, 1) RACB_GEMM_INST_TMA(kCordic, 16, kNT, 1)
RACB_GEMM_INST_TMA(kCordic, 16, kNN, 2) RACB_GEMM_INST_TMA(kCordic, 16, kNT, 2)
RACB_GEMM_INST_TMA(kCordic, 16, kNN, 3) RACB_GEMM_INST_TMA(kCordic, 16, kNT, 3)
RACB_GEMM_INST_TMA(kCordic, 16, kNN, 4) RACB_GEMM_INST_TMA(kCordic, 16, kNT, 4)
}
