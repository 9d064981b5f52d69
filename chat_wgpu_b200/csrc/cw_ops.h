// cw_ops.h -- host-side launchers of the op kernels, shared with the model.
#pragma once
#include "cw_common.h"

namespace cw {

int launch_rmsnorm(cw_ctx* ctx, const float* x, const float* w, float* y, int rows, int dim,
                   float eps, int unit);
int launch_rope(cw_ctx* ctx, const float* x, float* y, int rows, int hd, int pos, float theta);
// Split count for a key span over n_kv heads (about two CTAs per SM).
int attention_splits(cw_ctx* ctx, int span, int n_kv);
// k/v addressed as base + kv_head*head_stride + j*row_stride (floats).
int launch_attention(cw_ctx* ctx, const float* q, const float* k, const float* v, float* out,
                     int n_heads, int n_kv, int seq, int hd, float softcap, int window,
                     long head_stride, long row_stride, int n_splits, float* part);

}  // namespace cw
