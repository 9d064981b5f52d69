// Persistent step kernel for head_dim 32, GQA group <= 4, GEMV config 0 for
// K = dim and 0 for K = n_heads * head_dim (see the variant table in cw_step.cu).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_1_4_0_0() { return k_step<1, 4, 0, 0>; }

}  // namespace cw
