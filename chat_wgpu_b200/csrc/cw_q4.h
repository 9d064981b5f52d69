// cw_q4.h -- host-side launchers shared between the op entry points and the
// model code.
#pragma once
#include "cw_common.h"

namespace cw {

// y[N] = W x for a Q4 weight in LAYOUT (cw_device.cuh), enqueued on ctx->stream.
template <int LAYOUT>
int launch_q4_gemv(cw_ctx* ctx, const float* x, const void* payload, const void* scales, int K,
                   long N, float* y);

// Repack device GGUF Q4_0 blocks of a [rows, in_f] tensor into a new
// persistent packed weight buffer (payload plane, then f16 scale plane).
int pack_q4_0(cw_ctx* ctx, const void* d_src, size_t rows, size_t in_f, cw_buf* out);

}  // namespace cw
