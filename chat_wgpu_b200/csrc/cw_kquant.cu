// cw_kquant.cu -- GEMV and exact dequantisation over GGUF k-quant weights
// (Q4_K, Q5_K, Q6_K super-blocks of 256 weights), kept in HBM as the raw
// GGUF blocks.
//
// Q6_K follows the reference's dequant_q6_k (src/loader/dequant.rs:102-131):
// w = (d * sc) * (q - 32), f32, left to right.  Q4_K / Q5_K are not in the
// reference (dequant.rs:6, ROADMAP.md:52-53); they restate ggml's published
// block_q4_K / block_q5_K layout: w = (d * sc) * q - (dmin * m).  Each
// formula is evaluated in the stated order with one f32 rounding per
// operation (no contraction), so dequantised values are exact to it.
//
// GEMV: one warp per output row; the 32 lanes split each super-block 8
// weights apiece (Q4_K/Q5_K lane l: 64-weight chunk l/8, 4 bytes of nibbles
// at 4*(l%8) -> 4 low-nibble and 4 high-nibble weights; Q6_K lane t: half
// t/16, weights l, l+1 (l = 2*(t%16)) at offsets 0/32/64/96 of the half),
// x staged once per CTA in shared memory, f32 accumulation, warp reduction.
#include <stdint.h>

#include "cw_common.h"
#include "cw_device.cuh"

namespace cw {

template <int T>
struct KQ;
template <>
struct KQ<CW_GGUF_Q4_K> {
    static constexpr int BYTES = 144;
};
template <>
struct KQ<CW_GGUF_Q5_K> {
    static constexpr int BYTES = 176;
};
template <>
struct KQ<CW_GGUF_Q6_K> {
    static constexpr int BYTES = 210;
};

__device__ __forceinline__ float kq_f16(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__device__ __forceinline__ void kq_scale_min(int j, const uint8_t* q, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// The 8 weights lane `lane` owns in super-block `blk`: values w[8] and their
// indices within the block idx[8].
template <int T>
__device__ __forceinline__ void kq_lane(const uint8_t* __restrict__ blk, int lane, float (&w)[8],
                                        int (&idx)[8]) {
    if constexpr (T == CW_GGUF_Q6_K) {
        const int h = lane >> 4, l0 = 2 * (lane & 15), is = l0 >> 4;
        const uint8_t* ql = blk + 64 * h;
        const uint8_t* qh = blk + 128 + 32 * h;
        const int8_t* sc = (const int8_t*)(blk + 192 + 8 * h);
        const float d = kq_f16(blk + 208);
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int l = l0 + u;
            const int a = ql[l], b = ql[l + 32], hb = qh[l];
            const int q1 = ((a & 0x0f) | (((hb >> 0) & 3) << 4)) - 32;
            const int q2 = ((b & 0x0f) | (((hb >> 2) & 3) << 4)) - 32;
            const int q3 = ((a >> 4) | (((hb >> 4) & 3) << 4)) - 32;
            const int q4 = ((b >> 4) | (((hb >> 6) & 3) << 4)) - 32;
            w[4 * u + 0] = __fmul_rn(__fmul_rn(d, (float)sc[is + 0]), (float)q1);
            w[4 * u + 1] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2]), (float)q2);
            w[4 * u + 2] = __fmul_rn(__fmul_rn(d, (float)sc[is + 4]), (float)q3);
            w[4 * u + 3] = __fmul_rn(__fmul_rn(d, (float)sc[is + 6]), (float)q4);
            idx[4 * u + 0] = 128 * h + l;
            idx[4 * u + 1] = 128 * h + l + 32;
            idx[4 * u + 2] = 128 * h + l + 64;
            idx[4 * u + 3] = 128 * h + l + 96;
        }
    } else {
        constexpr bool five = T == CW_GGUF_Q5_K;
        const int c = lane >> 3, j0 = 4 * (lane & 7);
        const float d = kq_f16(blk), dmin = kq_f16(blk + 2);
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + (five ? 48 : 16) + 32 * c + j0;
        int sc1, m1, sc2, m2;
        kq_scale_min(2 * c, scales, &sc1, &m1);
        kq_scale_min(2 * c + 1, scales, &sc2, &m2);
        const float d1 = __fmul_rn(d, (float)sc1), mm1 = __fmul_rn(dmin, (float)m1);
        const float d2 = __fmul_rn(d, (float)sc2), mm2 = __fmul_rn(dmin, (float)m2);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int lo = qs[i] & 0x0f, hi = qs[i] >> 4;
            if constexpr (five) {
                const int hb = blk[16 + j0 + i];
                lo += ((hb >> (2 * c)) & 1) << 4;
                hi += ((hb >> (2 * c + 1)) & 1) << 4;
            }
            w[i] = __fsub_rn(__fmul_rn(d1, (float)lo), mm1);
            w[4 + i] = __fsub_rn(__fmul_rn(d2, (float)hi), mm2);
            idx[i] = 64 * c + j0 + i;
            idx[4 + i] = 64 * c + 32 + j0 + i;
        }
    }
}

template <int T>
__global__ void __launch_bounds__(256) k_kq_gemv(const uint8_t* __restrict__ wraw, int K, int N,
                                                 const float* __restrict__ x,
                                                 float* __restrict__ y) {
    extern __shared__ float xs[];
    constexpr int BYTES = KQ<T>::BYTES;
    for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = x[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nbk = K / 256;
    for (int r = blockIdx.x * 8 + warp; r < N; r += gridDim.x * 8) {
        const uint8_t* row = wraw + (size_t)r * nbk * BYTES;
        float acc = 0.f;
        for (int b = 0; b < nbk; b++) {
            float w[8];
            int idx[8];
            kq_lane<T>(row + (size_t)b * BYTES, lane, w, idx);
            const float* xb = xs + 256 * b;
#pragma unroll
            for (int i = 0; i < 8; i++) acc = fmaf(w[i], xb[idx[i]], acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) y[r] = acc;
    }
}

template <int T>
__global__ void k_kq_dequant(const uint8_t* __restrict__ wraw, long n_blocks,
                             float* __restrict__ out) {
    constexpr int BYTES = KQ<T>::BYTES;
    const long n = n_blocks * 32;  // one item per (block, lane)
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const long b = i >> 5;
        float w[8];
        int idx[8];
        kq_lane<T>(wraw + b * BYTES, (int)(i & 31), w, idx);
#pragma unroll
        for (int k = 0; k < 8; k++) out[b * 256 + idx[k]] = w[k];
    }
}

int kq_block_bytes(int type) {
    switch (type) {
        case CW_GGUF_Q4_K: return 144;
        case CW_GGUF_Q5_K: return 176;
        case CW_GGUF_Q6_K: return 210;
        default: return 0;
    }
}

}  // namespace cw

using namespace cw;

extern "C" {

int cw_kquant_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, int type, size_t in_f, size_t out_f,
                   cw_buf* out) {
    clear_error();
    const int bb = kq_block_bytes(type);
    CW_CHECK(ctx && out && bb, CW_ERR_INVALID_ARG, "cw_kquant_gemv: bad arguments (type %d)",
             type);
    CW_CHECK(in_f % 256 == 0 && in_f > 0 && in_f <= 16384 && out_f > 0 && out_f < (1u << 31),
             CW_ERR_INVALID_ARG, "cw_kquant_gemv: bad shape [%zu, %zu] (in_f %% 256, <= 16384)",
             out_f, in_f);
    BufEntry *ex, *ew, *ey;
    CW_TRY(buf_get(ctx, x, &ex, in_f * 4, "cw_kquant_gemv(x)"));
    CW_TRY(buf_get(ctx, w, &ew, out_f * (in_f / 256) * bb, "cw_kquant_gemv(w)"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, out_f, out, &ey));
    ex = &ctx->bufs[x];
    ew = &ctx->bufs[w];
    const int grid = (int)std::min<size_t>((out_f + 7) / 8, (size_t)ctx->sm_count * 8);
    const size_t smem = in_f * 4;
    OpScope scope(ctx, "kquant_gemv");
    auto go = [&](auto kern) -> int {
        if (smem > 48 * 1024)
            CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        kern<<<grid, 256, smem, ctx->stream>>>((const uint8_t*)ew->ptr, (int)in_f, (int)out_f,
                                               (const float*)ex->ptr, (float*)ey->ptr);
        return check_launch("kquant gemv");
    };
    if (type == CW_GGUF_Q4_K) return go(k_kq_gemv<CW_GGUF_Q4_K>);
    if (type == CW_GGUF_Q5_K) return go(k_kq_gemv<CW_GGUF_Q5_K>);
    return go(k_kq_gemv<CW_GGUF_Q6_K>);
}

int cw_kquant_dequant(cw_ctx* ctx, cw_buf w, int type, size_t rows, size_t in_f, cw_buf* out) {
    clear_error();
    const int bb = kq_block_bytes(type);
    CW_CHECK(ctx && out && bb && in_f % 256 == 0 && in_f > 0 && rows > 0, CW_ERR_INVALID_ARG,
             "cw_kquant_dequant: bad arguments");
    BufEntry *ew, *eo;
    CW_TRY(buf_get(ctx, w, &ew, rows * (in_f / 256) * bb, "cw_kquant_dequant(w)"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, rows * in_f, out, &eo));
    ew = &ctx->bufs[w];
    const long nb = (long)(rows * (in_f / 256));
    const int grid = (int)std::min<long>((nb * 32 + 255) / 256, (long)ctx->sm_count * 16);
    OpScope scope(ctx, "kquant_dequant");
    const uint8_t* src = (const uint8_t*)ew->ptr;
    float* dst = (float*)eo->ptr;
    if (type == CW_GGUF_Q4_K)
        k_kq_dequant<CW_GGUF_Q4_K><<<grid, 256, 0, ctx->stream>>>(src, nb, dst);
    else if (type == CW_GGUF_Q5_K)
        k_kq_dequant<CW_GGUF_Q5_K><<<grid, 256, 0, ctx->stream>>>(src, nb, dst);
    else
        k_kq_dequant<CW_GGUF_Q6_K><<<grid, 256, 0, ctx->stream>>>(src, nb, dst);
    return check_launch("kquant dequant");
}

}  // extern "C"
