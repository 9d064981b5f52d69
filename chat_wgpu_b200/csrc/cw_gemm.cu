// cw_gemm.cu -- the tcgen05 prefill GEMM kernel (design notes and device
// primitives in cw_gemm.cuh), the operand-split kernels, TMA tensor maps,
// launch, and the cw_q4_0_gemm op.
#include <cudaTypedefs.h>

#include <mutex>

#include "cw_common.h"
#include "cw_gemm.cuh"

namespace cw {

__global__ void __launch_bounds__(192, 1)
    k_gemm_x3(const __grid_constant__ CUtensorMap tXh, const __grid_constant__ CUtensorMap tXl,
              const __grid_constant__ CUtensorMap tWh, const __grid_constant__ CUtensorMap tWl,
              GemmArgs a) {
    extern __shared__ uint8_t gm_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)gm_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = (uint64_t*)(sm + (size_t)GM_ST * GM_STAGE);
    uint64_t* empty = full + GM_ST;
    uint64_t* done = empty + GM_ST;
    uint32_t* tslot = (uint32_t*)(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (a.M + GM_BM - 1) / GM_BM, n_tiles = (a.N + GM_BN - 1) / GM_BN;
    int mt, nt;
    const int ks = blockIdx.x % a.ksplit;  // this CTA's K range
    gm_tile(blockIdx.x / a.ksplit, m_tiles, n_tiles, a.group_m, &mt, &nt);
    const int m0 = mt * GM_BM, n0 = nt * GM_BN;
    const int KB_all = (a.K + GM_BK - 1) / GM_BK;
    const int per = (KB_all + a.ksplit - 1) / a.ksplit;
    const int kb0 = min(KB_all, ks * per);
    const int KB = min(KB_all, kb0 + per) - kb0;  // K steps of this CTA (>= 1 by the host's choice)
    const bool partial = a.ksplit > 1;
    float* const ybase = partial ? a.ws + (size_t)ks * a.M * a.N : a.y;
    const int ldy = partial ? a.N : a.ldy;
    const float* const bias = partial ? nullptr : a.bias;
    const int epi = partial ? GE_STORE : a.epi;

    if (threadIdx.x == 0) {
        for (int s = 0; s < GM_ST; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tXh);
        tma_prefetch_desc(&tXl);
        tma_prefetch_desc(&tWh);
        tma_prefetch_desc(&tWl);
    }
    if (warp == 1) tmem_alloc(tslot, GM_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            int kb = 0;
            for (; kb < KB; kb++) {
                const int s = kb % GM_ST;
                if (kb >= GM_ST && !mbar_wait(&empty[s], ((kb / GM_ST) - 1) & 1, GM_WAIT_NS)) {
                    gm_fail(a.status);
                    break;
                }
                uint8_t* st = sm + (size_t)s * GM_STAGE;
                mbar_expect_tx(&full[s], GM_STAGE);
                const int kx = (kb0 + kb) * GM_BK;
                tma_load_2d(st, &tXh, kx, m0, &full[s]);
                tma_load_2d(st + GM_TILE, &tXl, kx, m0, &full[s]);
                tma_load_2d(st + 2 * GM_TILE, &tWh, kx, n0, &full[s]);
                tma_load_2d(st + 3 * GM_TILE, &tWl, kx, n0, &full[s]);
            }
            // copies still in flight land before the CTA may exit
            for (int j = max(0, kb - GM_ST); j < kb; j++)
                if (!mbar_wait(&full[j % GM_ST], (j / GM_ST) & 1, GM_WAIT_NS)) gm_fail(a.status);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            constexpr uint32_t idesc = umma_idesc_f16(GM_BM, GM_BN);
            const uint32_t acc_hi = tmem, acc_lo = tmem + GM_BN;
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % GM_ST;
                if (!mbar_wait(&full[s], (kb / GM_ST) & 1, GM_WAIT_NS)) {
                    gm_fail(a.status);
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_addr(sm + (size_t)s * GM_STAGE);
                const uint64_t dxh = umma_desc_sw128(st), dxl = umma_desc_sw128(st + GM_TILE);
                const uint64_t dwh = umma_desc_sw128(st + 2 * GM_TILE),
                               dwl = umma_desc_sw128(st + 3 * GM_TILE);
#pragma unroll
                for (int k = 0; k < GM_BK / 16; k++) {
                    const uint64_t adv = (uint64_t)(k * 32) >> 4;  // 16 f16 = 32 bytes along K
                    const uint32_t first = (kb > 0 || k > 0) ? 1u : 0u;
                    umma_f16(acc_hi, dxh + adv, dwh + adv, idesc, first);
                    umma_f16(acc_lo, dxh + adv, dwl + adv, idesc, first);
                    umma_f16(acc_lo, dxl + adv, dwh + adv, idesc, 1u);
                }
                tc_commit(&empty[s]);  // stage reusable once these MMAs have read it
            }
            tc_commit(done);  // also on the error path: the drain waits for in-flight MMAs
        }
    } else {  // ---- epilogue: warps 2..5
        const bool ok = mbar_wait(done, 0, GM_WAIT_NS);
        if (!ok) gm_fail(a.status);
        tc_fence_after();
        const int q = warp & 3;
        const int row = m0 + q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
        for (int c = 0; c < GM_BN; c += 16) {
            uint32_t h[16], l[16];
            tmem_ld16(lane_base + c, h);
            tmem_ld16(lane_base + GM_BN + c, l);
            tmem_wait_ld();
            if (!ok || row >= a.M) continue;
            float* yr = ybase + (size_t)row * ldy;
            const int nb = n0 + c;
            if (nb + 16 <= a.N && (ldy & 3) == 0) {
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    float r[4];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        r[t] = __uint_as_float(h[j + t]) +
                               __uint_as_float(l[j + t]) * (1.0f / GM_LO);
                        if (bias) r[t] += bias[nb + j + t];
                    }
                    float4* dst = (float4*)(yr + nb + j);
                    if (epi == GE_ADD) {
                        const float4 o = *dst;
                        r[0] += o.x;
                        r[1] += o.y;
                        r[2] += o.z;
                        r[3] += o.w;
                    }
                    *dst = make_float4(r[0], r[1], r[2], r[3]);
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    if (nb + j >= a.N) continue;
                    float acc =
                        __uint_as_float(h[j]) + __uint_as_float(l[j]) * (1.0f / GM_LO);
                    if (bias) acc += bias[nb + j];
                    if (epi == GE_ADD) acc += yr[nb + j];
                    yr[nb + j] = acc;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, GM_TMEM_COLS);
    }
}

// Split-K: y (=|+=) bias + sum of the ksplit partial tiles, in split order
// (deterministic).
__global__ void k_gemm_reduce(const float* __restrict__ ws, int ksplit, int M, int N,
                              float* __restrict__ y, int ldy, const float* __restrict__ bias,
                              int epi) {
    const long n = (long)M * N;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / N), c = (int)(i - (long)r * N);
        float acc = ws[i];
        for (int k = 1; k < ksplit; k++) acc += ws[(size_t)k * n + i];
        if (bias) acc += bias[c];
        float* dst = y + (size_t)r * ldy + c;
        *dst = epi == GE_ADD ? *dst + acc : acc;
    }
}

// Packed Q4_0 [rows, K] -> Wh, Wl f16 [rows, K] (row-major, K contiguous).
// One thread per 8 consecutive weights (one 16-byte chunk of each output).
// GGUF block layout (dequant.rs:62-78): byte j holds weight j (low nibble)
// and weight j+16 (high nibble); w = (q - 8) * d is exact in f32.
__global__ void k_q4_split(const uint8_t* __restrict__ payload, const __half* __restrict__ scales,
                           long rows, int K, __half* __restrict__ wh, __half* __restrict__ wl) {
    const int nb = K / 32;
    const long chunks = rows * (long)(K / 8);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < chunks;
         i += (long)gridDim.x * blockDim.x) {
        const long r = i / (K / 8);
        const int c = (int)(i - r * (K / 8));
        const int b = c >> 2, sub = c & 3;
        const long blk = r * nb + b;
        const float d = __half2float(scales[blk]);
        const uint2 raw = *(const uint2*)(payload + blk * 16 + (sub & 1) * 8);
        const uint32_t w2[2] = {raw.x, raw.y};
        __align__(16) __half hv[8], lv[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            uint32_t byte = (w2[j >> 2] >> ((j & 3) * 8)) & 0xff;
            int q = (sub < 2) ? (int)(byte & 0xf) : (int)(byte >> 4);
            float w = __fmul_rn(d, (float)(q - 8));
            __half h = __float2half_rn(w);
            hv[j] = h;
            lv[j] = __float2half_rn((w - __half2float(h)) * GM_LO);
        }
        const long o = r * (long)K + (long)c * 8;
        *(uint4*)(wh + o) = *(const uint4*)hv;
        *(uint4*)(wl + o) = *(const uint4*)lv;
    }
}

// X f32 [M, K] (row stride ldx) -> Xh, Xl f16 [M, K].
__global__ void k_x_split(const float* __restrict__ x, long M, int K, int ldx,
                          __half* __restrict__ xh, __half* __restrict__ xl) {
    const long n = M * (long)(K / 4);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const long r = i / (K / 4);
        const int c = (int)(i - r * (K / 4)) * 4;
        const float4 v = *(const float4*)(x + r * ldx + c);
        __align__(8) __half hv[4], lv[4];
        split_f16(v.x, &hv[0], &lv[0]);
        split_f16(v.y, &hv[1], &lv[1]);
        split_f16(v.z, &hv[2], &lv[2]);
        split_f16(v.w, &hv[3], &lv[3]);
        *(uint2*)(xh + r * K + c) = *(const uint2*)hv;
        *(uint2*)(xl + r * K + c) = *(const uint2*)lv;
    }
}

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
            int N, int K, float* y, int ldy, const float* bias, int epi, float* ws,
            size_t ws_bytes) {
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
    // split K until about two CTAs per SM are busy (each split >= 2 K steps),
    // as far as the workspace holds the partial tiles
    const int KB = (K + GM_BK - 1) / GM_BK;
    int ks = 1;
    if (ws)
        while (m_tiles * n_tiles * ks * 2 < 2 * ctx->sm_count && ks * 2 <= KB / 2 && ks < 32 &&
               (size_t)(ks * 2) * M * N * 4 <= ws_bytes)
            ks *= 2;
    a.ksplit = ks;
    a.ws = ws;
    k_gemm_x3<<<m_tiles * n_tiles * ks, 192, GM_SMEM, ctx->stream>>>(m_xh, m_xl, m_wh, m_wl, a);
    CW_TRY(check_launch("gemm_x3"));
    if (ks == 1) return CW_OK;
    const long n = (long)M * N;
    const int grid = (int)std::min<long>((n + 255) / 256, (long)ctx->sm_count * 8);
    k_gemm_reduce<<<grid, 256, 0, ctx->stream>>>(ws, ks, M, N, y, ldy, bias, epi);
    return check_launch("gemm split-K reduce");
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
    const size_t wsbytes = 32ull << 20;  // split-K partials (short M)
    uint8_t* sc = nullptr;
    CW_TRY(gemm_scratch(ctx, 2 * xbytes + 2 * wbytes + wsbytes, &sc));
    uint8_t *xh = sc, *xl = sc + xbytes, *wh = sc + 2 * xbytes, *wl = wh + wbytes;
    float* ws = (float*)(wl + wbytes);
    OpScope scope(ctx, "q4_gemm");
    {
        OpScope s1(ctx, "q4_gemm.split_x");
        CW_TRY(x_split(ctx, (const float*)ex->ptr, (long)rows, (int)in_f, (int)in_f, xh, xl));
    }
    {
        OpScope s2(ctx, "q4_gemm.split_w");
        CW_TRY(q4_split(ctx, ew->ptr, (const char*)ew->ptr + ew->scale_off, (long)out_f,
                        (int)in_f, wh, wl));
    }
    OpScope s3(ctx, "q4_gemm.mma");
    return gemm_x3(ctx, xh, xl, wh, wl, (int)rows, (int)out_f, (int)in_f, (float*)ey->ptr,
                   (int)out_f, nullptr, GE_STORE, ws, wsbytes);
}

}  // extern "C"
