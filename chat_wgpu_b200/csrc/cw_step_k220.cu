// Persistent step kernel for head_dim 64, GQA group <= 2 and GEMV config 0
// for K = dim (the variant table is in cw_step.cu; small test shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_2_2_0_0() { return k_step<2, 2, 0, false>; }

}  // namespace cw
