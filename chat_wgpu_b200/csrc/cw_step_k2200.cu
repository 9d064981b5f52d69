// Persistent step kernel for head_dim 64, GQA group <= 2, GEMV config 0 for
// K = dim and 0 for K = n_heads * head_dim (see the variant table in cw_step.cu).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_2_2_0_0() { return k_step<2, 2, 0, 0>; }

}  // namespace cw
