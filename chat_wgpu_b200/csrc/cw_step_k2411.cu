// Persistent step kernel for head_dim 64, GQA group <= 4, GEMV config 1 for
// K = dim and 1 for K = n_heads * head_dim (see the variant table in cw_step.cu).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_2_4_1_1() { return k_step<2, 4, 1, 1>; }

}  // namespace cw
