// cw_kquant.cu -- GEMV and exact dequantisation over raw GGUF weights kept
// in HBM as the file's blocks: the k-quants and F32 / F16 / BF16 / Q8_0 /
// Q4_1 (formats and device code in cw_kquant.cuh).
//
// GEMV: Q4_K / Q5_K (raw super-blocks), Q6_K and Q8_0 (the aligned splits of
// cw_q6_k_split / cw_q8_0_split) run on the streaming GEMV of cw_gemv.cuh:
// weights streamed
// through shared memory, integer dp4a products against q24 activation
// planes.  The per-row kernel below serves the other types and Q6_K in its
// raw form: one warp per output row; the 32 lanes split each super-block 8
// weights apiece (Q4_K/Q5_K lane l: 64-weight chunk l/8, 4 bytes of nibbles
// at 4*(l%8) -> 4 low-nibble and 4 high-nibble weights; Q6_K lane t: half
// t/16, weights l, l+1 (l = 2*(t%16)) at offsets 0/32/64/96 of the half),
// x staged once per CTA in shared memory, f32 accumulation, warp reduction.
#include "cw_gemv.cuh"
#include "cw_kquant.cuh"

namespace cw {

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
        int b = 0;
        for (; b + KQ_UNROLL <= nbk; b += KQ_UNROLL) {
            KqRaw<T> raw[KQ_UNROLL];
#pragma unroll
            for (int u = 0; u < KQ_UNROLL; u++) raw[u] = kq_load<T>(row + (size_t)(b + u) * BYTES, lane);
#pragma unroll
            for (int u = 0; u < KQ_UNROLL; u++) acc = kq_dot<T>(raw[u], xs + 256 * (b + u), lane, acc);
        }
        for (; b < nbk; b++) acc = kq_dot<T>(kq_load<T>(row + (size_t)b * BYTES, lane), xs + 256 * b, lane, acc);
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

// One warp per super-block: the 210-byte block is 2-byte aligned, so it is
// moved as 105 half-words (104 to the payload plane, the last one is d).
__global__ void k_q6k_split(const uint8_t* __restrict__ raw, long nsb, uint8_t* __restrict__ pay,
                            __half* __restrict__ d) {
    const int lane = threadIdx.x & 31;
    const long w0 = (blockIdx.x * (long)blockDim.x + threadIdx.x) >> 5;
    const long nw = ((long)gridDim.x * blockDim.x) >> 5;
    for (long s = w0; s < nsb; s += nw) {
        const uint16_t* src = reinterpret_cast<const uint16_t*>(raw + s * 210);
        uint16_t* dst = reinterpret_cast<uint16_t*>(pay + s * 208);
        for (int i = lane; i < 104; i += 32) dst[i] = src[i];
        if (lane == 0) d[s] = __ushort_as_half(src[104]);
    }
}

int q6k_split(cw_ctx* ctx, const uint8_t* raw, size_t nsb, uint8_t* pay, __half* d) {
    if (!nsb) return CW_OK;
    const int grid = (int)std::min<size_t>((nsb + 7) / 8, (size_t)ctx->sm_count * 16);
    k_q6k_split<<<grid, 256, 0, ctx->stream>>>(raw, (long)nsb, pay, d);
    return check_launch("q6_k split");
}

// One thread per 34-byte block (2-byte aligned): d to the scale plane, the
// 32 codes to one 32-byte payload row.
__global__ void k_q8_split(const uint8_t* __restrict__ raw, long nb, uint8_t* __restrict__ pay,
                           __half* __restrict__ d) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= nb) return;
    const uint16_t* s = reinterpret_cast<const uint16_t*>(raw + i * 34);
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; k++) w[k] = (uint32_t)s[1 + 2 * k] | ((uint32_t)s[2 + 2 * k] << 16);
    d[i] = __ushort_as_half(s[0]);
    uint4* p = reinterpret_cast<uint4*>(pay + i * 32);
    p[0] = make_uint4(w[0], w[1], w[2], w[3]);
    p[1] = make_uint4(w[4], w[5], w[6], w[7]);
}

int q8_split(cw_ctx* ctx, const uint8_t* raw, size_t nb, uint8_t* pay, __half* d) {
    if (!nb) return CW_OK;
    k_q8_split<<<(unsigned)((nb + 255) / 256), 256, 0, ctx->stream>>>(raw, (long)nb, pay, d);
    return check_launch("q8_0 split");
}

int kq_block_bytes(int type) {
    switch (type) {
        case CW_GGUF_Q4_K: return KQ<CW_GGUF_Q4_K>::BYTES;
        case CW_GGUF_Q5_K: return KQ<CW_GGUF_Q5_K>::BYTES;
        case CW_GGUF_Q6_K: return KQ<CW_GGUF_Q6_K>::BYTES;
        case CW_GGUF_F32: return KQ<CW_GGUF_F32>::BYTES;
        case CW_GGUF_F16: return KQ<CW_GGUF_F16>::BYTES;
        case CW_GGUF_BF16: return KQ<CW_GGUF_BF16>::BYTES;
        case CW_GGUF_Q8_0: return KQ<CW_GGUF_Q8_0>::BYTES;
        case CW_GGUF_Q4_1: return KQ<CW_GGUF_Q4_1>::BYTES;
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
    OpScope scope(ctx, "kquant_gemv");
    if ((type == CW_GGUF_Q4_K || type == CW_GGUF_Q5_K) && sgemv_supported(LAYOUT_Q4K, (int)in_f)) {
        GemvArgs a = {};
        a.payload = (const uint8_t*)ew->ptr;
        a.K = (int)in_f;
        a.N = (int)out_f;
        a.x = (const float*)ex->ptr;
        a.y = (float*)ey->ptr;
        return launch_sgemv(ctx, type == CW_GGUF_Q4_K ? LAYOUT_Q4K : LAYOUT_Q5K, PRO_X, EPI_STORE,
                            a, false);
    }
    const int grid = (int)std::min<size_t>((out_f + 7) / 8, (size_t)ctx->sm_count * 8);
    const size_t smem = in_f * 4;
    auto go = [&](auto kern) -> int {
        if (smem > 48 * 1024)
            CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        kern<<<grid, 256, smem, ctx->stream>>>((const uint8_t*)ew->ptr, (int)in_f, (int)out_f,
                                               (const float*)ex->ptr, (float*)ey->ptr);
        return check_launch("kquant gemv");
    };
    switch (type) {
        case CW_GGUF_Q4_K: return go(k_kq_gemv<CW_GGUF_Q4_K>);
        case CW_GGUF_Q5_K: return go(k_kq_gemv<CW_GGUF_Q5_K>);
        case CW_GGUF_F32: return go(k_kq_gemv<CW_GGUF_F32>);
        case CW_GGUF_F16: return go(k_kq_gemv<CW_GGUF_F16>);
        case CW_GGUF_BF16: return go(k_kq_gemv<CW_GGUF_BF16>);
        case CW_GGUF_Q8_0: return go(k_kq_gemv<CW_GGUF_Q8_0>);
        case CW_GGUF_Q4_1: return go(k_kq_gemv<CW_GGUF_Q4_1>);
        default: return go(k_kq_gemv<CW_GGUF_Q6_K>);
    }
}

int cw_q6_k_split(cw_ctx* ctx, cw_buf w, size_t rows, size_t in_f, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out && rows > 0 && in_f % 256 == 0 && in_f > 0, CW_ERR_INVALID_ARG,
             "cw_q6_k_split: bad arguments");
    const size_t nsb = rows * (in_f / 256);
    BufEntry *ew, *eo;
    CW_TRY(buf_get(ctx, w, &ew, nsb * 210, "cw_q6_k_split(w)"));
    cudaSetDevice(ctx->device);
    CW_TRY(buf_new(ctx, nsb * 210, BUF_PERSISTENT, out, &eo));
    ew = &ctx->bufs[w];
    eo->q6k_split = true;
    eo->rows = rows;
    eo->in_f = in_f;
    eo->scale_off = nsb * 208;
    uint8_t* base = (uint8_t*)eo->ptr;
    return q6k_split(ctx, (const uint8_t*)ew->ptr, nsb, base, (__half*)(base + nsb * 208));
}

int cw_q6_k_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, size_t in_f, size_t out_f, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out && out_f > 0 && out_f < (1u << 31), CW_ERR_INVALID_ARG,
             "cw_q6_k_gemv: bad arguments");
    CW_CHECK(sgemv_supported(LAYOUT_Q6K, (int)in_f), CW_ERR_UNSUPPORTED,
             "cw_q6_k_gemv: in_f=%zu not handled (a multiple of 256, at most 24576)", in_f);
    BufEntry *ex, *ew, *ey;
    CW_TRY(buf_get(ctx, x, &ex, in_f * 4, "cw_q6_k_gemv(x)"));
    CW_TRY(buf_get(ctx, w, &ew, 0, "cw_q6_k_gemv(w)"));
    CW_CHECK(ew->q6k_split && ew->rows == out_f && ew->in_f == in_f, CW_ERR_INVALID_ARG,
             "cw_q6_k_gemv: buffer %llu is not a split Q6_K weight of [%zu, %zu]",
             (unsigned long long)w, out_f, in_f);
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, out_f, out, &ey));
    ex = &ctx->bufs[x];
    ew = &ctx->bufs[w];
    OpScope scope(ctx, "kquant_gemv");
    GemvArgs a = {};
    a.payload = (const uint8_t*)ew->ptr;
    a.scales = (const char*)ew->ptr + ew->scale_off;
    a.K = (int)in_f;
    a.N = (int)out_f;
    a.x = (const float*)ex->ptr;
    a.y = (float*)ey->ptr;
    return launch_sgemv(ctx, LAYOUT_Q6K, PRO_X, EPI_STORE, a, false);
}

int cw_q8_0_split(cw_ctx* ctx, cw_buf w, size_t rows, size_t in_f, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out && rows > 0 && in_f % 32 == 0 && in_f > 0, CW_ERR_INVALID_ARG,
             "cw_q8_0_split: bad arguments");
    const size_t nb = rows * (in_f / 32);
    BufEntry *ew, *eo;
    CW_TRY(buf_get(ctx, w, &ew, nb * 34, "cw_q8_0_split(w)"));
    cudaSetDevice(ctx->device);
    CW_TRY(buf_new(ctx, nb * 34, BUF_PERSISTENT, out, &eo));
    ew = &ctx->bufs[w];
    eo->q8_split = true;
    eo->rows = rows;
    eo->in_f = in_f;
    eo->scale_off = nb * 32;
    uint8_t* base = (uint8_t*)eo->ptr;
    return q8_split(ctx, (const uint8_t*)ew->ptr, nb, base, (__half*)(base + nb * 32));
}

int cw_q8_0_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, size_t in_f, size_t out_f, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out && out_f > 0 && out_f < (1u << 31), CW_ERR_INVALID_ARG,
             "cw_q8_0_gemv: bad arguments");
    CW_CHECK(sgemv_supported(LAYOUT_Q8, (int)in_f), CW_ERR_UNSUPPORTED,
             "cw_q8_0_gemv: in_f=%zu not handled (a multiple of 256, at most 24576)", in_f);
    BufEntry *ex, *ew, *ey;
    CW_TRY(buf_get(ctx, x, &ex, in_f * 4, "cw_q8_0_gemv(x)"));
    CW_TRY(buf_get(ctx, w, &ew, 0, "cw_q8_0_gemv(w)"));
    CW_CHECK(ew->q8_split && ew->rows == out_f && ew->in_f == in_f, CW_ERR_INVALID_ARG,
             "cw_q8_0_gemv: buffer %llu is not a split Q8_0 weight of [%zu, %zu]",
             (unsigned long long)w, out_f, in_f);
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, out_f, out, &ey));
    ex = &ctx->bufs[x];
    ew = &ctx->bufs[w];
    OpScope scope(ctx, "kquant_gemv");
    GemvArgs a = {};
    a.payload = (const uint8_t*)ew->ptr;
    a.scales = (const char*)ew->ptr + ew->scale_off;
    a.K = (int)in_f;
    a.N = (int)out_f;
    a.x = (const float*)ex->ptr;
    a.y = (float*)ey->ptr;
    return launch_sgemv(ctx, LAYOUT_Q8, PRO_X, EPI_STORE, a, false);
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
#define CW_KQ_DEQ(T) k_kq_dequant<T><<<grid, 256, 0, ctx->stream>>>(src, nb, dst)
    switch (type) {
        case CW_GGUF_Q4_K: CW_KQ_DEQ(CW_GGUF_Q4_K); break;
        case CW_GGUF_Q5_K: CW_KQ_DEQ(CW_GGUF_Q5_K); break;
        case CW_GGUF_F32: CW_KQ_DEQ(CW_GGUF_F32); break;
        case CW_GGUF_F16: CW_KQ_DEQ(CW_GGUF_F16); break;
        case CW_GGUF_BF16: CW_KQ_DEQ(CW_GGUF_BF16); break;
        case CW_GGUF_Q8_0: CW_KQ_DEQ(CW_GGUF_Q8_0); break;
        case CW_GGUF_Q4_1: CW_KQ_DEQ(CW_GGUF_Q4_1); break;
        default: CW_KQ_DEQ(CW_GGUF_Q6_K); break;
    }
#undef CW_KQ_DEQ
    return check_launch("kquant dequant");
}

}  // extern "C"
