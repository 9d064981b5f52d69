// Persistent step kernel for head_dim 32, GQA group <= 4 and GEMV config 0
// for K = dim (the variant table is in cw_step.cu; small test shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_1_4_0_0() { return k_step<1, 4, 0, false>; }

}  // namespace cw
