// Persistent step kernel for head_dim 128, GQA group <= 2 and GEMV config 0
// for K = dim (the variant table is in cw_step.cu; Qwen3-0.6B shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_4_2_0_0() { return k_step<4, 2, 0, false>; }

}  // namespace cw
