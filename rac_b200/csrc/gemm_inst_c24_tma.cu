// CORDIC GEMM, n = 24 iterations unrolled, TMA-staged: NN and NT, tiles 1-4.
#include "gemm_kernel.cuh"
namespace racb {
RACB_GEMM_INST_TMA(kCordic, 24, kNN, 1) RACB_GEMM_INST_TMA(kCordic, 24, kNT, 1)
RACB_GEMM_INST_TMA(kCordic, 24, kNN, 2) RACB_GEMM_INST_TMA(kCordic, 24, kNT, 2)
RACB_GEMM_INST_TMA(kCordic, 24, kNN, 3) RACB_GEMM_INST_TMA(kCordic, 24, kNT, 3)
RACB_GEMM_INST_TMA(kCordic, 24, kNN, 4) RACB_GEMM_INST_TMA(kCordic, 24, kNT, 4)
}
