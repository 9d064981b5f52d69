// cw_mgemv.h -- host interface of the co-batched decode GEMV (cw_mgemv.cu):
// Y[s] = W X[s] for every session s of a session group, Q4_0 weights
// streamed from HBM once for all of them.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "cw_common.h"

namespace cw {

struct MgArgs {
    const uint8_t* payload;  // GGUF Q4_0 nibble plane [N][K/32][16]
    const __half* scales;    // [N][K/32]
    int K, N;
    int B;                   // sessions of the group (rows of X and Y)
    // PRO_X: X rows [B][ldx] are the GEMV inputs.  PRO_NORM: they are the
    // residual H, and the input of session s is rmsnorm(H[s]) * gain(norm_w)
    // (norm.wgsl:20-56; unit: 1 + w).
    const float* x;
    int ldx;
    const float* norm_w;
    float eps;
    int unit;
    // output rows [B][ldy]: EPI_STORE y = Wx (+ bias), EPI_RESID y += Wx,
    // EPI_GLU y[i] = act(gate_i) * up_i over interleaved rows (2i gate, 2i+1 up)
    float* y;
    int ldy;
    const float* bias;
    int geglu;
    int* status;  // device status word (bounded waits report DEV_TIMEOUT)
    // K <= 4096: run the products on the integer tensor cores (mma.sync
    // m16n8k32) instead of dp4a; the integer sums are the same.  They read
    // the weight's tile-interleaved copy (mg_tile_pack).
    int mma;
    const uint8_t* tiles;
    // EPI_HEAD (integer-MMA path): logits cap * tanh(l / cap) (softcap > 0)
    // stored to yrow[s][row], and each session's argmax key (ties to the
    // lowest row, argmax.wgsl) atomicMax'ed into keys[s]
    float* const* yrow;
    unsigned long long* keys;
    float softcap;
};

// The tile-interleaved copy of a Q4_0 matrix the integer-MMA products read:
// per 16-row tile its payload [block][row][16 B], then its scales
// [block][row] (rows past the end zero).  Bytes for `rows` x K, and the
// packing kernel (enqueued on ctx->stream).
size_t mg_tile_bytes(int rows, int K);
int mg_tile_pack(cw_ctx* ctx, const uint8_t* payload, const __half* scales, int rows, int K,
                 void* dst);

// Whether the co-batched GEMV takes K for a group of B sessions (K/32 a
// multiple of 8 and at most 384 blocks; 1 <= B <= 8).
bool mgemv_supported(int K, int B);
// Launch on ctx->stream (pro: PRO_X / PRO_NORM, epi: EPI_STORE / EPI_RESID /
// EPI_GLU / EPI_HEAD of cw_gemv.cuh).
int launch_mgemv(cw_ctx* ctx, int pro, int epi, const MgArgs& a, bool pdl);

}  // namespace cw
