// Persistent step kernel for head_dim 128, GQA group <= 2 and GEMV config 1
// for K = dim (the variant table is in cw_step.cu; Qwen3-1.7B shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_4_2_1_0() { return k_step<4, 2, 1, false>; }

}  // namespace cw
