// CORDIC GEMM with a run-time iteration count: any n in [1, 24], any shape
// and alignment, every layout.  Bit-identical to the fixed-n kernels.
#include "gemm_kernel.cuh"
namespace racb {
#define L(LAY) RACB_GEMM_INST(kCordic, 0, LAY, 1, true) RACB_GEMM_INST(kCordic, 0, LAY, 1, false) \
               RACB_GEMM_INST(kCordic, 0, LAY, 3, true) RACB_GEMM_INST(kCordic, 0, LAY, 3, false)
L(kNN) L(kNT) L(kTN)
}
