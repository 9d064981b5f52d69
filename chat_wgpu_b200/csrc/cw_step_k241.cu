// Persistent step kernel for head_dim 64, GQA group <= 4 and GEMV config 1
// for K = dim (the variant table is in cw_step.cu; Llama-3.2-1B-like shapes).
#include "cw_step.cuh"

namespace cw {

StepKernel step_kernel_2_4_1_0() { return k_step<2, 4, 1, false>; }

}  // namespace cw
