// Persistent step kernel for head_dim 256, GQA group <= 2, GEMV config 2 for
// K = dim and the post-norm residual (the variant table is in cw_step.cu;
// Gemma-2-2B/9B shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_8_2_2_1() { return k_step<8, 2, 2, true>; }

}  // namespace cw
