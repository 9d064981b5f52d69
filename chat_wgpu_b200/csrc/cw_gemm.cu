// cw_gemm.cu -- host side of the tcgen05 prefill GEMM (kernels in
// cw_gemm.cuh): TMA tensor maps, operand splitting, launch, and the
// cw_q4_0_gemm op.
#include <cudaTypedefs.h>

#include <mutex>

#include "cw_common.h"
#include "cw_gemm.cuh"

namespace cw {

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
    });
    return fn;
}

// f16 [rows, K] row-major, box 64 (K) x 128 (rows), 128-byte swizzle: the
// canonical K-major operand layout the MMA descriptors expect.
static int tmap_f16(CUtensorMap* map, const void* base, long rows, int K) {
    auto enc = tmap_encode_fn();
    CW_CHECK(enc, CW_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    CW_CHECK(((uintptr_t)base & 15) == 0 && K % 8 == 0, CW_ERR_INVALID_ARG,
             "gemm operand must be 16-byte aligned with K %% 8 == 0");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)GM_BK, (cuuint32_t)GM_BM};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CW_CHECK(r == CUDA_SUCCESS, CW_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CW_OK;
}

int gemm_x3(cw_ctx* ctx, const void* xh, const void* xl, const void* wh, const void* wl, int M,
            int N, int K, float* y, int ldy, const float* bias, int epi) {
    CW_CHECK(M > 0 && N > 0 && K > 0 && K % 32 == 0 && ldy >= N, CW_ERR_INVALID_ARG,
             "gemm: bad shape M=%d N=%d K=%d ldy=%d", M, N, K, ldy);
    CUtensorMap m_xh, m_xl, m_wh, m_wl;
    CW_TRY(tmap_f16(&m_xh, xh, M, K));
    CW_TRY(tmap_f16(&m_xl, xl, M, K));
    CW_TRY(tmap_f16(&m_wh, wh, N, K));
    CW_TRY(tmap_f16(&m_wl, wl, N, K));
    static bool attr_set[64] = {};
    if (!attr_set[ctx->device & 63]) {
        CW_CUDA(cudaFuncSetAttribute(k_gemm_x3, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GM_SMEM));
        attr_set[ctx->device & 63] = true;
    }
    GemmArgs a{};
    a.y = y;
    a.bias = bias;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ldy = ldy;
    a.epi = epi;
    a.group_m = 8;
    a.status = ctx->d_status;
    const int m_tiles = (M + GM_BM - 1) / GM_BM, n_tiles = (N + GM_BN - 1) / GM_BN;
    k_gemm_x3<<<m_tiles * n_tiles, 192, GM_SMEM, ctx->stream>>>(m_xh, m_xl, m_wh, m_wl, a);
    return check_launch("gemm_x3");
}

int q4_split(cw_ctx* ctx, const void* payload, const void* scales, long rows, int K, void* wh,
             void* wl) {
    const long chunks = rows * (K / 8);
    const int grid = (int)std::min<long>((chunks + 255) / 256, (long)ctx->sm_count * 16);
    k_q4_split<<<grid, 256, 0, ctx->stream>>>((const uint8_t*)payload, (const __half*)scales, rows,
                                              K, (__half*)wh, (__half*)wl);
    return check_launch("q4_split");
}

int x_split(cw_ctx* ctx, const float* x, long M, int K, int ldx, void* xh, void* xl) {
    CW_CHECK(K % 4 == 0 && ldx % 4 == 0, CW_ERR_INVALID_ARG, "x_split: K and ldx must be %% 4");
    const long n = M * (K / 4);
    const int grid = (int)std::min<long>((n + 255) / 256, (long)ctx->sm_count * 16);
    k_x_split<<<grid, 256, 0, ctx->stream>>>(x, M, K, ldx, (__half*)xh, (__half*)xl);
    return check_launch("x_split");
}

static int gemm_scratch(cw_ctx* ctx, size_t bytes, uint8_t** p) {
    if (ctx->gemm_scratch_bytes < bytes) {
        CW_CUDA(cudaStreamSynchronize(ctx->stream));
        if (ctx->gemm_scratch) cudaFree(ctx->gemm_scratch);
        ctx->gemm_scratch = nullptr;
        ctx->gemm_scratch_bytes = 0;
        CW_CUDA(cudaMalloc(&ctx->gemm_scratch, bytes));
        ctx->gemm_scratch_bytes = bytes;
    }
    *p = (uint8_t*)ctx->gemm_scratch;
    return CW_OK;
}

}  // namespace cw

using namespace cw;

extern "C" {

int cw_q4_0_gemm(cw_ctx* ctx, cw_buf x, cw_buf w, size_t rows, size_t in_f, size_t out_f,
                 cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_q4_0_gemm: bad arguments");
    CW_CHECK(rows > 0 && rows < (1u << 30) && in_f % 32 == 0 && in_f > 0 && in_f < (1u << 30) &&
                 out_f > 0 && out_f < (1u << 30),
             CW_ERR_INVALID_ARG, "cw_q4_0_gemm: bad shape [%zu, %zu] x [%zu, %zu]^T", rows, in_f,
             out_f, in_f);
    BufEntry *ex, *ew, *ey;
    CW_TRY(buf_get(ctx, x, &ex, rows * in_f * 4, "cw_q4_0_gemm(x)"));
    CW_TRY(buf_get(ctx, w, &ew, 0, "cw_q4_0_gemm(w)"));
    CW_CHECK(ew->q4_0 && ew->rows == out_f && ew->in_f == in_f, CW_ERR_INVALID_ARG,
             "cw_q4_0_gemm(w): not a packed Q4_0 weight of shape [%zu, %zu]", out_f, in_f);
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, rows * out_f, out, &ey));
    ex = &ctx->bufs[x];
    ew = &ctx->bufs[w];
    const size_t xbytes = (rows * in_f * 2 + 255) / 256 * 256;
    const size_t wbytes = (out_f * in_f * 2 + 255) / 256 * 256;
    uint8_t* sc = nullptr;
    CW_TRY(gemm_scratch(ctx, 2 * xbytes + 2 * wbytes, &sc));
    uint8_t *xh = sc, *xl = sc + xbytes, *wh = sc + 2 * xbytes, *wl = wh + wbytes;
    OpScope scope(ctx, "q4_gemm");
    CW_TRY(x_split(ctx, (const float*)ex->ptr, (long)rows, (int)in_f, (int)in_f, xh, xl));
    CW_TRY(q4_split(ctx, ew->ptr, (const char*)ew->ptr + ew->scale_off, (long)out_f, (int)in_f,
                    wh, wl));
    return gemm_x3(ctx, xh, xl, wh, wl, (int)rows, (int)out_f, (int)in_f, (float*)ey->ptr,
                   (int)out_f, nullptr, GE_STORE);
}

}  // extern "C"
