// cw_ops.h -- host-side launchers of the op kernels, shared with the model.
#pragma once
#include "cw_common.h"

namespace cw {

int launch_rmsnorm(cw_ctx* ctx, const float* x, const float* w, float* y, int rows, int dim,
                   float eps, int unit);
int launch_rope(cw_ctx* ctx, const float* x, float* y, int rows, int hd, int pos, float theta);
// Split count for a key span over n_kv heads (about two CTAs per SM).
int attention_splits(cw_ctx* ctx, int span, int n_kv);
int attention_splits_for(int sm_count, int span, int n_kv);
// The attention launch with the stream, the split partials and the zeroed
// per-kv-head counters given explicitly (no context).
int launch_attention_raw(cudaStream_t st, const float* q, const float* k, const float* v,
                         float* out, int n_heads, int n_kv, int seq, int hd, float softcap,
                         int window, long head_stride, long row_stride, int n_splits, float* part,
                         unsigned* counters);
// k/v addressed as base + kv_head*head_stride + j*row_stride (floats).
int launch_attention(cw_ctx* ctx, const float* q, const float* k, const float* v, float* out,
                     int n_heads, int n_kv, int seq, int hd, float softcap, int window,
                     long head_stride, long row_stride, int n_splits, float* part);

}  // namespace cw
