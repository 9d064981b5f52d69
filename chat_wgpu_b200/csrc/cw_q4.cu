// cw_q4.cu -- Q4 GEMV entry points (chat-wgpu src/kernels/q4.rs), the GGUF
// Q4_0 pack/dequant kernels and the on-device re-quantiser.
#include <algorithm>
#include <map>
#include <vector>

#include "cw_common.h"
#include "cw_device.cuh"
#include "cw_gemv.cuh"
#include "cw_q4.h"

namespace cw {

// ---------------------------------------------------------------------------
// Stand-alone GEMV: every CTA converts x to q24 planes once, then walks row
// groups (8 warps x R rows) grid-stride.  The warp's lanes stride the K blocks
// of its R rows with 16-byte streaming loads; a warp-shuffle sum finishes each
// row.
// ---------------------------------------------------------------------------
template <int LAYOUT, int R>
__global__ void __launch_bounds__(256) k_q4_gemv(const float* __restrict__ x,
                                                 const uint8_t* __restrict__ payload,
                                                 const void* __restrict__ scales, int K, long N,
                                                 float* __restrict__ y) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int nb = K / 32;
    Q24 s = q24_carve(smem, nb);
    q24_prepare<LAYOUT>(s, x);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long groups = (N + 8 * R - 1) / (8 * R);
    for (long g = blockIdx.x; g < groups; g += gridDim.x) {
        long row0 = (g * 8 + warp) * R;
        if (row0 >= N) continue;
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = 0.f;
        q4_rows_dot<LAYOUT, R>(s, payload, scales, row0, N, lane, acc);
#pragma unroll
        for (int r = 0; r < R; r++) {
            float v = warp_sum(acc[r]);
            if (lane == r && row0 + r < N) y[row0 + r] = v;
        }
    }
}

template <int LAYOUT, int R>
static int launch_gemv_r(cw_ctx* ctx, const float* x, const void* payload, const void* scales,
                         int K, long N, float* y) {
    size_t smem = q24_bytes(K / 32);
    auto kern = k_q4_gemv<LAYOUT, R>;
    // occupancy per (device, smem size) of this instantiation, queried once
    static thread_local std::map<std::pair<int, size_t>, int> occ;
    auto key = std::make_pair(ctx->device, smem);
    auto it = occ.find(key);
    int per_sm = 0;
    if (it == occ.end()) {
        if (smem > 48 * 1024) {
            CW_CHECK((int)smem <= ctx->max_smem_optin, CW_ERR_UNSUPPORTED,
                     "q4 gemv: in_f=%d needs %zu bytes of shared memory", K, smem);
            CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        }
        CW_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem));
        per_sm = std::max(per_sm, 1);
        occ[key] = per_sm;
    } else {
        per_sm = it->second;
    }
    long groups = (N + 8 * R - 1) / (8 * R);
    long grid = std::min<long>(groups, (long)ctx->sm_count * per_sm);
    kern<<<(unsigned)grid, 256, smem, ctx->stream>>>(x, (const uint8_t*)payload, scales, K, N, y);
    return check_launch("q4 gemv");
}

template <int LAYOUT>
int launch_q4_gemv(cw_ctx* ctx, const float* x, const void* payload, const void* scales, int K,
                   long N, float* y) {
    if (sgemv_supported(LAYOUT, K)) {
        GemvArgs a = {};
        a.payload = (const uint8_t*)payload;
        a.scales = scales;
        a.K = K;
        a.N = (int)N;
        a.x = x;
        a.y = y;
        return launch_sgemv(ctx, LAYOUT, PRO_X, EPI_STORE, a, false);
    }
    // R rows per warp: 4 when there are enough rows to fill every SM twice
    // over, else fewer rows per warp and more warps.
    long sm2 = 2L * ctx->sm_count * 8;
    if (N >= sm2 * 4) return launch_gemv_r<LAYOUT, 4>(ctx, x, payload, scales, K, N, y);
    if (N >= sm2 * 2) return launch_gemv_r<LAYOUT, 2>(ctx, x, payload, scales, K, N, y);
    return launch_gemv_r<LAYOUT, 1>(ctx, x, payload, scales, K, N, y);
}
template int launch_q4_gemv<LAYOUT_GGUF>(cw_ctx*, const float*, const void*, const void*, int,
                                         long, float*);
template int launch_q4_gemv<LAYOUT_REF>(cw_ctx*, const float*, const void*, const void*, int, long,
                                        float*);

// ---------------------------------------------------------------------------
// GGUF Q4_0 repack: block i (18 bytes: f16 d, 16 nibble bytes) -> payload[i]
// (16 bytes) and scales[i] (2 bytes).  Pure byte moves: lossless.
// ---------------------------------------------------------------------------
__global__ void k_q4_0_pack(const uint8_t* __restrict__ src, size_t nblocks,
                            uint8_t* __restrict__ payload, uint16_t* __restrict__ scales) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src + i * 18);  // 2-byte aligned
    uint32_t w[4];
#pragma unroll
    for (int k = 0; k < 4; k++) w[k] = (uint32_t)s[1 + 2 * k] | ((uint32_t)s[2 + 2 * k] << 16);
    scales[i] = s[0];
    reinterpret_cast<uint4*>(payload)[i] = make_uint4(w[0], w[1], w[2], w[3]);
}

// Exact dequantisation (dequant.rs:62-78): d * (q - 8) is exact in f32.
__global__ void k_q4_0_dequant(const uint8_t* __restrict__ payload,
                               const uint16_t* __restrict__ scales, size_t nblocks,
                               float* __restrict__ out) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nblocks) return;
    float d = __half2float(__ushort_as_half(scales[i]));
    uint4 q = reinterpret_cast<const uint4*>(payload)[i];
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
    float* o = out + i * 32;
#pragma unroll
    for (int j = 0; j < 16; j++) {
        uint32_t byte = (w[j >> 2] >> (8 * (j & 3))) & 0xff;
        o[j] = __fmul_rn(d, (float)((int)(byte & 0xf) - 8));
        o[j + 16] = __fmul_rn(d, (float)((int)(byte >> 4) - 8));
    }
}

// q4.rs:37-60 on the device, one thread per (row, block).  1.0f/d and the
// product v*inv are IEEE round-to-nearest, roundf rounds half away from zero
// like Rust's f32::round, and the float->int conversion saturates with NaN ->
// 0 like Rust's `as i32`; the results are bit-identical to the host routine.
__global__ void k_q4_quantize(const float* __restrict__ w, size_t rows, int in_f,
                              float* __restrict__ scales, uint32_t* __restrict__ quants) {
    const int nb = in_f / 32;
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * (size_t)nb) return;
    size_t o = i / nb, b = i % nb;
    const float* v = w + o * in_f + b * 32;
    float absmax = 0.f;
    for (int j = 0; j < 32; j++) absmax = fmaxf(absmax, fabsf(v[j]));
    float d = __fdiv_rn(absmax, 8.0f);
    float inv = (d != 0.f) ? __fdiv_rn(1.0f, d) : 0.f;
    scales[o * nb + b] = d;
    for (int wd = 0; wd < 4; wd++) {
        uint32_t word = 0;
        for (int n = 0; n < 8; n++) {
            float r = roundf(__fmul_rn(v[wd * 8 + n], inv));
            int qi = (int)((unsigned)__float2int_rz(r) + 8u);
            qi = qi < 0 ? 0 : (qi > 15 ? 15 : qi);
            word |= (uint32_t)qi << (n * 4);
        }
        quants[o * (in_f / 8) + b * 4 + wd] = word;
    }
}

int pack_q4_0(cw_ctx* ctx, const void* d_src, size_t rows, size_t in_f, cw_buf* out) {
    size_t nblocks = rows * (in_f / 32);
    size_t pay = nblocks * 16;
    size_t scale_off = (pay + 255) & ~size_t(255);
    BufEntry* e;
    CW_TRY(buf_new(ctx, scale_off + nblocks * 2, BUF_PERSISTENT, out, &e));
    e->q4_0 = true;
    e->rows = rows;
    e->in_f = in_f;
    e->scale_off = scale_off;
    if (nblocks) {
        unsigned grid = (unsigned)((nblocks + 255) / 256);
        k_q4_0_pack<<<grid, 256, 0, ctx->stream>>>(
            (const uint8_t*)d_src, nblocks, (uint8_t*)e->ptr,
            (uint16_t*)((char*)e->ptr + scale_off));
        CW_TRY(check_launch("q4_0 pack"));
    }
    return CW_OK;
}

static int q4_0_weight(cw_ctx* ctx, cw_buf w, size_t rows, size_t in_f, BufEntry** e,
                       const char* what) {
    CW_TRY(buf_get(ctx, w, e, 0, what));
    CW_CHECK((*e)->q4_0, CW_ERR_INVALID_ARG, "%s: buffer %llu is not a packed Q4_0 weight", what,
             (unsigned long long)w);
    CW_CHECK((*e)->rows == rows && (*e)->in_f == in_f, CW_ERR_INVALID_ARG,
             "%s: weight is [%zu, %zu], call says [%zu, %zu]", what, (*e)->rows, (*e)->in_f, rows,
             in_f);
    return CW_OK;
}

}  // namespace cw

using namespace cw;

extern "C" {

int cw_q4_gemv(cw_ctx* ctx, cw_buf x, cw_buf scales, cw_buf quants, size_t in_f, size_t out_f,
               cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_q4_gemv: bad arguments");
    CW_CHECK(in_f % 32 == 0 && in_f > 0, CW_ERR_INVALID_ARG,
             "q4 expects in_f multiple of 32 (got %zu)", in_f);
    CW_CHECK(out_f > 0 && out_f < (1ull << 31), CW_ERR_INVALID_ARG, "cw_q4_gemv: bad out_f %zu",
             out_f);
    BufEntry *ex, *es, *eq, *ey;
    CW_TRY(buf_get(ctx, x, &ex, in_f * 4, "cw_q4_gemv(x)"));
    CW_TRY(buf_get(ctx, scales, &es, out_f * in_f / 32 * 4, "cw_q4_gemv(scales)"));
    CW_TRY(buf_get(ctx, quants, &eq, out_f * in_f / 8 * 4, "cw_q4_gemv(quants)"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, out_f, out, &ey));
    OpScope scope(ctx, "q4_gemv");
    return launch_q4_gemv<LAYOUT_REF>(ctx, (const float*)ex->ptr, eq->ptr, es->ptr, (int)in_f,
                                      (long)out_f, (float*)ey->ptr);
}

int cw_q4_quantize(cw_ctx* ctx, cw_buf w, size_t out_f, size_t in_f, cw_buf* scales,
                   cw_buf* quants) {
    clear_error();
    CW_CHECK(ctx && scales && quants, CW_ERR_INVALID_ARG, "cw_q4_quantize: bad arguments");
    CW_CHECK(in_f % 32 == 0 && in_f > 0 && out_f > 0, CW_ERR_INVALID_ARG,
             "q4 expects in_f multiple of 32 (got %zu)", in_f);
    BufEntry *ew, *es, *eq;
    CW_TRY(buf_get(ctx, w, &ew, out_f * in_f * 4, "cw_q4_quantize(w)"));
    cudaSetDevice(ctx->device);
    CW_TRY(buf_new(ctx, out_f * in_f / 32 * 4, BUF_PERSISTENT, scales, &es));
    CW_TRY(buf_new(ctx, out_f * in_f / 8 * 4, BUF_PERSISTENT, quants, &eq));
    ew = &ctx->bufs[w];
    size_t n = out_f * (in_f / 32);
    OpScope scope(ctx, "q4_quantize");
    k_q4_quantize<<<(unsigned)((n + 127) / 128), 128, 0, ctx->stream>>>(
        (const float*)ew->ptr, out_f, (int)in_f, (float*)ctx->bufs[*scales].ptr,
        (uint32_t*)ctx->bufs[*quants].ptr);
    return check_launch("q4 quantize");
}

int cw_q4_0_upload(cw_ctx* ctx, const void* gguf_blocks, size_t rows, size_t in_f, cw_buf* w) {
    clear_error();
    CW_CHECK(ctx && w && gguf_blocks, CW_ERR_INVALID_ARG, "cw_q4_0_upload: bad arguments");
    CW_CHECK(in_f % 32 == 0 && in_f > 0 && rows > 0, CW_ERR_INVALID_ARG,
             "cw_q4_0_upload: in_f must be a positive multiple of 32 (got %zu)", in_f);
    cudaSetDevice(ctx->device);
    size_t nbytes = rows * (in_f / 32) * 18;
    void* tmp = nullptr;
    CW_CUDA(cudaMalloc(&tmp, nbytes));
    cudaError_t e = cudaMemcpyAsync(tmp, gguf_blocks, nbytes, cudaMemcpyHostToDevice, ctx->stream);
    int rc = (e == cudaSuccess) ? pack_q4_0(ctx, tmp, rows, in_f, w)
                                : set_error(CW_ERR_CUDA, "cw_q4_0_upload: %s", cudaGetErrorString(e));
    cudaStreamSynchronize(ctx->stream);
    cudaFree(tmp);
    return rc;
}

int cw_q4_0_pack(cw_ctx* ctx, cw_buf gguf_blocks, size_t rows, size_t in_f, cw_buf* w) {
    clear_error();
    CW_CHECK(ctx && w, CW_ERR_INVALID_ARG, "cw_q4_0_pack: bad arguments");
    CW_CHECK(in_f % 32 == 0 && in_f > 0 && rows > 0, CW_ERR_INVALID_ARG,
             "cw_q4_0_pack: in_f must be a positive multiple of 32 (got %zu)", in_f);
    BufEntry* s;
    CW_TRY(buf_get(ctx, gguf_blocks, &s, rows * (in_f / 32) * 18, "cw_q4_0_pack(src)"));
    cudaSetDevice(ctx->device);
    void* src = s->ptr;
    return pack_q4_0(ctx, src, rows, in_f, w);
}

int cw_q4_0_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, size_t in_f, size_t out_f, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_q4_0_gemv: bad arguments");
    CW_CHECK(in_f % 32 == 0 && in_f > 0 && out_f > 0 && out_f < (1ull << 31), CW_ERR_INVALID_ARG,
             "cw_q4_0_gemv: bad shape [%zu, %zu]", out_f, in_f);
    BufEntry *ex, *ew, *ey;
    CW_TRY(buf_get(ctx, x, &ex, in_f * 4, "cw_q4_0_gemv(x)"));
    CW_TRY(q4_0_weight(ctx, w, out_f, in_f, &ew, "cw_q4_0_gemv(w)"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, out_f, out, &ey));
    ex = &ctx->bufs[x];
    ew = &ctx->bufs[w];
    OpScope scope(ctx, "q4_gemv");
    return launch_q4_gemv<LAYOUT_GGUF>(ctx, (const float*)ex->ptr, ew->ptr,
                                       (const char*)ew->ptr + ew->scale_off, (int)in_f,
                                       (long)out_f, (float*)ey->ptr);
}

int cw_q4_0_gemv_bench(cw_ctx* ctx, cw_buf x, const cw_buf* ws, size_t n_w, size_t in_f,
                       size_t out_f, size_t iters, double* us_per_launch) {
    clear_error();
    CW_CHECK(ctx && ws && n_w > 0 && iters > 0 && us_per_launch, CW_ERR_INVALID_ARG,
             "cw_q4_0_gemv_bench: bad arguments");
    CW_CHECK(in_f % 32 == 0 && in_f > 0 && out_f > 0 && out_f < (1ull << 31), CW_ERR_INVALID_ARG,
             "cw_q4_0_gemv_bench: bad shape [%zu, %zu]", out_f, in_f);
    BufEntry *ex, *ey;
    CW_TRY(buf_get(ctx, x, &ex, in_f * 4, "cw_q4_0_gemv_bench(x)"));
    std::vector<BufEntry*> we(n_w);
    for (size_t i = 0; i < n_w; i++)
        CW_TRY(q4_0_weight(ctx, ws[i], out_f, in_f, &we[i], "cw_q4_0_gemv_bench(w)"));
    cudaSetDevice(ctx->device);
    cw_buf y;
    CW_TRY(arena_get(ctx, out_f, &y, &ey));
    // one untimed pass over every weight (attributes, first-touch)
    for (size_t i = 0; i < n_w; i++)
        CW_TRY(launch_q4_gemv<LAYOUT_GGUF>(ctx, (const float*)ex->ptr, we[i]->ptr,
                                           (const char*)we[i]->ptr + we[i]->scale_off, (int)in_f,
                                           (long)out_f, (float*)ey->ptr));
    // the launches are replayed as one CUDA graph so host launch overhead
    // does not starve the device between short kernels
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    CW_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
    int rc = CW_OK;
    for (size_t it = 0; it < iters && rc == CW_OK; it++) {
        BufEntry* w = we[it % n_w];
        rc = launch_q4_gemv<LAYOUT_GGUF>(ctx, (const float*)ex->ptr, w->ptr,
                                         (const char*)w->ptr + w->scale_off, (int)in_f,
                                         (long)out_f, (float*)ey->ptr);
    }
    cudaError_t ce = cudaStreamEndCapture(ctx->stream, &graph);
    if (rc != CW_OK) {
        if (graph) cudaGraphDestroy(graph);
        return rc;
    }
    if (ce != cudaSuccess) return set_error(CW_ERR_CUDA, "bench capture: %s", cudaGetErrorString(ce));
    ce = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ce != cudaSuccess)
        return set_error(CW_ERR_CUDA, "bench instantiate: %s", cudaGetErrorString(ce));
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaGraphLaunch(exec, ctx->stream);  // warm
    cudaEventRecord(e0, ctx->stream);
    cudaGraphLaunch(exec, ctx->stream);
    cudaEventRecord(e1, ctx->stream);
    ce = cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaGraphExecDestroy(exec);
    if (ce != cudaSuccess) return set_error(CW_ERR_CUDA, "bench: %s", cudaGetErrorString(ce));
    *us_per_launch = (double)ms * 1000.0 / (double)iters;
    return CW_OK;
}

int cw_q4_0_dequant(cw_ctx* ctx, cw_buf w, size_t rows, size_t in_f, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_q4_0_dequant: bad arguments");
    BufEntry *ew, *eo;
    CW_TRY(q4_0_weight(ctx, w, rows, in_f, &ew, "cw_q4_0_dequant(w)"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, rows * in_f, out, &eo));
    ew = &ctx->bufs[w];
    size_t nblocks = rows * (in_f / 32);
    OpScope scope(ctx, "q4_dequant");
    k_q4_0_dequant<<<(unsigned)((nblocks + 255) / 256), 256, 0, ctx->stream>>>(
        (const uint8_t*)ew->ptr, (const uint16_t*)((const char*)ew->ptr + ew->scale_off), nblocks,
        (float*)eo->ptr);
    return check_launch("q4_0 dequant");
}

}  // extern "C"
