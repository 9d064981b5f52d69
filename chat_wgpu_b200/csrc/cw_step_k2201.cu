// Persistent step kernel for head_dim 64, GQA group <= 2, GEMV config 0 for
// K = dim and the post-norm residual (the variant table is in cw_step.cu;
// the small Gemma-2 test shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_2_2_0_1() { return k_step<2, 2, 0, true>; }

}  // namespace cw
