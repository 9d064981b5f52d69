// Persistent step kernel for head_dim 128, GQA group <= 2, GEMV config 0 for
// K = dim and 1 for K = n_heads * head_dim (see the variant table in cw_step.cu).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_4_2_0_1() { return k_step<4, 2, 0, 1>; }

}  // namespace cw
