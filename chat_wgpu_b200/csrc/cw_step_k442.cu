// Persistent step kernel for head_dim 128, GQA group <= 4 and GEMV config 2
// for K = dim (the variant table is in cw_step.cu; Qwen3-4B/8B shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_4_4_2_0() { return k_step<4, 4, 2, false>; }

}  // namespace cw
