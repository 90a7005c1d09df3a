// SHIFTADD-mode GEMM instantiations (integer shift-add product, run-time n).
#include "gemm_kernel.cuh"
namespace racb {
#define L(LAY) RACB_GEMM_INST(kShiftAdd, 0, LAY, 1, true) RACB_GEMM_INST(kShiftAdd, 0, LAY, 1, false) \
               RACB_GEMM_INST(kShiftAdd, 0, LAY, 3, true) RACB_GEMM_INST(kShiftAdd, 0, LAY, 3, false)
L(kNN) L(kNT) L(kTN)
}
