// Persistent step kernel for head_dim 128, GQA group <= 4, GEMV config 2 for
// K = dim and 2 for K = n_heads * head_dim (see the variant table in cw_step.cu).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_4_4_2_2() { return k_step<4, 4, 2, 2>; }

}  // namespace cw
