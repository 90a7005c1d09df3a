// FAST-mode GEMM on packed FFMA2 with TMA staging (gemm_fast.cuh) instantiations.
#include "gemm_fast.cuh"
namespace racb {
RACB_FAST_TMA_INST(kNN, 1) RACB_FAST_TMA_INST(kTN, 1) RACB_FAST_TMA_INST(kNN, 2) RACB_FAST_TMA_INST(kTN, 2)
}
