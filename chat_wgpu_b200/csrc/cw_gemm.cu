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

// ---- Q4_0 dequantised in shared memory -------------------------------------------
// Packed GEMM layout of a Q4_0 weight (built once per weight): per 128-row
// tile and 64-wide K step one contiguous 4608-byte record, the 128 rows' two
// 16-byte GGUF payloads (bytes 0..4095, row-major) then their two f16 scales
// (4096..4607).  Rows past N and blocks past K/32 are zero (they dequantise
// to 0).  One cp.async.bulk moves a record.
constexpr int GQ_REC = GM_BN * 32 + GM_BN * 4;  // 4608 bytes
// Xh, Xl, Wh, Wl, raw record; stages 1024-byte aligned (128-byte swizzle atoms)
constexpr int GQ_STAGE = (4 * GM_TILE + GQ_REC + 1023) / 1024 * 1024;
constexpr size_t GQ_SMEM = (size_t)GM_ST * GQ_STAGE + 256 + 1024;

__global__ void k_q4_tile_pack(const uint8_t* __restrict__ payload,
                               const __half* __restrict__ scales, int rows, int K,
                               uint8_t* __restrict__ out) {
    const int nb = K / 32, KBp = (K + GM_BK - 1) / GM_BK;
    const long n_items = (long)rows * KBp;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n_items;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / KBp), kb = (int)(i - (long)r * KBp);
        uint8_t* rec = out + ((size_t)(r / GM_BN) * KBp + kb) * GQ_REC;
        const int rr = r % GM_BN;
        uint4 p0 = make_uint4(0, 0, 0, 0), p1 = p0;
        __half s0 = __float2half(0.f), s1 = s0;
        const int b0 = 2 * kb, b1 = 2 * kb + 1;
        p0 = *(const uint4*)(payload + ((size_t)r * nb + b0) * 16);
        s0 = scales[(size_t)r * nb + b0];
        if (b1 < nb) {
            p1 = *(const uint4*)(payload + ((size_t)r * nb + b1) * 16);
            s1 = scales[(size_t)r * nb + b1];
        }
        *(uint4*)(rec + rr * 32) = p0;
        *(uint4*)(rec + rr * 32 + 16) = p1;
        *(__half2*)(rec + GM_BN * 32 + rr * 4) = __halves2half2(s0, s1);
    }
}

// 8 weights of one 16-byte chunk: GGUF block byte j holds weight j (low
// nibble) and j + 16 (high nibble); chunk c of a 64-wide K step covers
// weights 8c .. 8c+7, i.e. block c/4, sub-range (c%4)*8.
__device__ __forceinline__ void gq_chunk(const uint2 bytes8, bool high, float d, uint4* hi,
                                         uint4* lo) {
    const uint32_t w2[2] = {bytes8.x, bytes8.y};
    __align__(16) __half hv[8], lv[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint32_t byte = (w2[j >> 2] >> ((j & 3) * 8)) & 0xffu;
        const int q = high ? (int)(byte >> 4) : (int)(byte & 0xfu);
        const float w = __fmul_rn(d, (float)(q - 8));  // exact
        const __half h = __float2half_rn(w);
        hv[j] = h;
        lv[j] = __float2half_rn((w - __half2float(h)) * GM_LO);
    }
    *hi = *(const uint4*)hv;
    *lo = *(const uint4*)lv;
}

// k_gemm_x3 with W read as packed Q4_0 records: warps 2-5 (one thread per W
// row) dequantise each stage's record into the swizzled f16 hi/lo tiles the
// MMA reads (the same values k_q4_split produces), then drain TMEM as the
// epilogue.  Streams 0.5625 bytes per weight instead of 4.
__global__ void __launch_bounds__(192, 1)
    k_gemm_q4(const __grid_constant__ CUtensorMap tXh, const __grid_constant__ CUtensorMap tXl,
              const uint8_t* __restrict__ wpack, GemmArgs a) {
    extern __shared__ uint8_t gm_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)gm_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* full = (uint64_t*)(sm + (size_t)GM_ST * GQ_STAGE);  // X tiles + raw record landed
    uint64_t* bfull = full + GM_ST;                                // W tiles written
    uint64_t* empty = bfull + GM_ST;                               // stage consumed by the MMAs
    uint64_t* done = empty + GM_ST;
    uint32_t* tslot = (uint32_t*)(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (a.M + GM_BM - 1) / GM_BM, n_tiles = (a.N + GM_BN - 1) / GM_BN;
    int mt, nt;
    const int ks = blockIdx.x % a.ksplit;
    gm_tile(blockIdx.x / a.ksplit, m_tiles, n_tiles, a.group_m, &mt, &nt);
    const int m0 = mt * GM_BM, n0 = nt * GM_BN;
    const int KB_all = (a.K + GM_BK - 1) / GM_BK;
    const int per = (KB_all + a.ksplit - 1) / a.ksplit;
    const int kb0 = min(KB_all, ks * per);
    const int KB = min(KB_all, kb0 + per) - kb0;
    const bool partial = a.ksplit > 1;
    float* const ybase = partial ? a.ws + (size_t)ks * a.M * a.N : a.y;
    const int ldy = partial ? a.N : a.ldy;
    const float* const bias = partial ? nullptr : a.bias;
    const int epi = partial ? GE_STORE : a.epi;
    const uint8_t* wtile = wpack + ((size_t)nt * KB_all + kb0) * GQ_REC;

    if (threadIdx.x == 0) {
        for (int s = 0; s < GM_ST; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&bfull[s], 128);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tXh);
        tma_prefetch_desc(&tXl);
    }
    if (warp == 1) tmem_alloc(tslot, GM_TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA / bulk producer
            int kb = 0;
            for (; kb < KB; kb++) {
                const int s = kb % GM_ST;
                if (kb >= GM_ST && !mbar_wait(&empty[s], ((kb / GM_ST) - 1) & 1, GM_WAIT_NS)) {
                    gm_fail(a.status);
                    break;
                }
                uint8_t* st = sm + (size_t)s * GQ_STAGE;
                mbar_expect_tx(&full[s], 2 * GM_TILE + GQ_REC);
                const int kx = (kb0 + kb) * GM_BK;
                tma_load_2d(st, &tXh, kx, m0, &full[s]);
                tma_load_2d(st + GM_TILE, &tXl, kx, m0, &full[s]);
                bulk_g2s(st + 4 * GM_TILE, wtile + (size_t)kb * GQ_REC, GQ_REC, &full[s]);
            }
            for (int j = max(0, kb - GM_ST); j < kb; j++)
                if (!mbar_wait(&full[j % GM_ST], (j / GM_ST) & 1, GM_WAIT_NS)) gm_fail(a.status);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            constexpr uint32_t idesc = umma_idesc_f16(GM_BM, GM_BN);
            const uint32_t acc_hi = tmem, acc_lo = tmem + GM_BN;
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % GM_ST;
                if (!mbar_wait(&full[s], (kb / GM_ST) & 1, GM_WAIT_NS) ||
                    !mbar_wait(&bfull[s], (kb / GM_ST) & 1, GM_WAIT_NS)) {
                    gm_fail(a.status);
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_addr(sm + (size_t)s * GQ_STAGE);
                const uint64_t dxh = umma_desc_sw128(st), dxl = umma_desc_sw128(st + GM_TILE);
                const uint64_t dwh = umma_desc_sw128(st + 2 * GM_TILE),
                               dwl = umma_desc_sw128(st + 3 * GM_TILE);
#pragma unroll
                for (int k = 0; k < GM_BK / 16; k++) {
                    const uint64_t adv = (uint64_t)(k * 32) >> 4;
                    const uint32_t first = (kb > 0 || k > 0) ? 1u : 0u;
                    umma_f16(acc_hi, dxh + adv, dwh + adv, idesc, first);
                    umma_f16(acc_lo, dxh + adv, dwl + adv, idesc, first);
                    umma_f16(acc_lo, dxl + adv, dwh + adv, idesc, 1u);
                }
                tc_commit(&empty[s]);
            }
            tc_commit(done);
        }
    } else {  // ---- warps 2..5: dequantise W records, then the epilogue
        const int t = threadIdx.x - 64;  // W row within the tile
        bool ok = true;
        for (int kb = 0; kb < KB && ok; kb++) {
            const int s = kb % GM_ST;
            if (!mbar_wait(&full[s], (kb / GM_ST) & 1, GM_WAIT_NS)) {
                gm_fail(a.status);
                ok = false;
                break;
            }
            uint8_t* st = sm + (size_t)s * GQ_STAGE;
            const uint8_t* rec = st + 4 * GM_TILE;
            const uint4 pay0 = *(const uint4*)(rec + t * 32);
            const uint4 pay1 = *(const uint4*)(rec + t * 32 + 16);
            const __half2 sc = *(const __half2*)(rec + GM_BN * 32 + t * 4);
            const float d0 = __low2float(sc), d1 = __high2float(sc);
            uint8_t* wh = st + 2 * GM_TILE + t * 128;
            uint8_t* wl = st + 3 * GM_TILE + t * 128;
            const int sw = t & 7;
#pragma unroll
            for (int c = 0; c < 8; c++) {
                const uint4 pay = c < 4 ? pay0 : pay1;
                const int sub = c & 3;
                const uint2 b8 = (sub & 1) ? make_uint2(pay.z, pay.w) : make_uint2(pay.x, pay.y);
                uint4 h, l;
                gq_chunk(b8, sub >= 2, c < 4 ? d0 : d1, &h, &l);
                *(uint4*)(wh + ((c ^ sw) << 4)) = h;
                *(uint4*)(wl + ((c ^ sw) << 4)) = l;
            }
            fence_proxy_async();  // generic-proxy stores -> visible to the MMA's async proxy
            mbar_arrive(&bfull[s]);
        }
        const bool ok_done = mbar_wait(done, 0, GM_WAIT_NS);
        if (!ok_done) gm_fail(a.status);
        ok = ok && ok_done;
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
                    for (int u = 0; u < 4; u++) {
                        r[u] = __uint_as_float(h[j + u]) +
                               __uint_as_float(l[j + u]) * (1.0f / GM_LO);
                        if (bias) r[u] += bias[nb + j + u];
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
                    float acc = __uint_as_float(h[j]) + __uint_as_float(l[j]) * (1.0f / GM_LO);
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

size_t q4_tile_bytes(int rows, int K) {
    return (size_t)((rows + GM_BN - 1) / GM_BN) * ((K + GM_BK - 1) / GM_BK) * GQ_REC;
}

int q4_tile_pack(cw_ctx* ctx, const void* payload, const void* scales, int rows, int K,
                 void* out) {
    CW_CUDA(cudaMemsetAsync(out, 0, q4_tile_bytes(rows, K), ctx->stream));
    const long items = (long)rows * ((K + GM_BK - 1) / GM_BK);
    const int grid = (int)std::min<long>((items + 255) / 256, (long)ctx->sm_count * 16);
    k_q4_tile_pack<<<grid, 256, 0, ctx->stream>>>((const uint8_t*)payload, (const __half*)scales,
                                                  rows, K, (uint8_t*)out);
    return check_launch("q4_tile_pack");
}

int gemm_q4(cw_ctx* ctx, const void* xh, const void* xl, const void* wpack, int M, int N, int K,
            float* y, int ldy, const float* bias, int epi, float* ws, size_t ws_bytes) {
    CW_CHECK(M > 0 && N > 0 && K > 0 && K % 32 == 0 && ldy >= N, CW_ERR_INVALID_ARG,
             "gemm: bad shape M=%d N=%d K=%d ldy=%d", M, N, K, ldy);
    CW_CHECK(((uintptr_t)wpack & 15) == 0, CW_ERR_INVALID_ARG, "gemm: packed W not 16-byte aligned");
    CUtensorMap m_xh, m_xl;
    CW_TRY(tmap_f16(&m_xh, xh, M, K));
    CW_TRY(tmap_f16(&m_xl, xl, M, K));
    static bool attr_set[64] = {};
    if (!attr_set[ctx->device & 63]) {
        CW_CUDA(cudaFuncSetAttribute(k_gemm_q4, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GQ_SMEM));
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
    const int KB = (K + GM_BK - 1) / GM_BK;
    int ks = 1;
    if (ws)
        while (m_tiles * n_tiles * ks * 2 < 2 * ctx->sm_count && ks * 2 <= KB / 2 && ks < 32 &&
               (size_t)(ks * 2) * M * N * 4 <= ws_bytes)
            ks *= 2;
    a.ksplit = ks;
    a.ws = ws;
    k_gemm_q4<<<m_tiles * n_tiles * ks, 192, GQ_SMEM, ctx->stream>>>(
        m_xh, m_xl, (const uint8_t*)wpack, a);
    CW_TRY(check_launch("gemm_q4"));
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
    // rows > 256: W split once into its f16 pair, streamed by k_gemm_x3 (the
    // MMA pipe is the bound); rows <= 256: packed Q4_0 records dequantised in
    // shared memory by k_gemm_q4, with split-K partials
    const bool big = rows > 256;
    const size_t xbytes = (rows * in_f * 2 + 255) / 256 * 256;
    const size_t wbytes = big ? 2 * ((out_f * in_f * 2 + 255) / 256 * 256)
                              : (q4_tile_bytes((int)out_f, (int)in_f) + 255) / 256 * 256;
    const size_t wsbytes = big ? 0 : 32ull << 20;
    uint8_t* sc = nullptr;
    CW_TRY(gemm_scratch(ctx, 2 * xbytes + wbytes + wsbytes, &sc));
    uint8_t *xh = sc, *xl = sc + xbytes, *wp = sc + 2 * xbytes;
    float* ws = (float*)(wp + wbytes);
    const char* scales = (const char*)ew->ptr + ew->scale_off;
    OpScope scope(ctx, "q4_gemm");
    {
        OpScope s1(ctx, "q4_gemm.split_x");
        CW_TRY(x_split(ctx, (const float*)ex->ptr, (long)rows, (int)in_f, (int)in_f, xh, xl));
    }
    {
        OpScope s2(ctx, "q4_gemm.prep_w");
        if (big)
            CW_TRY(q4_split(ctx, ew->ptr, scales, (long)out_f, (int)in_f, wp, wp + wbytes / 2));
        else
            CW_TRY(q4_tile_pack(ctx, ew->ptr, scales, (int)out_f, (int)in_f, wp));
    }
    OpScope s3(ctx, "q4_gemm.mma");
    if (big)
        return gemm_x3(ctx, xh, xl, wp, wp + wbytes / 2, (int)rows, (int)out_f, (int)in_f,
                       (float*)ey->ptr, (int)out_f, nullptr, GE_STORE);
    return gemm_q4(ctx, xh, xl, wp, (int)rows, (int)out_f, (int)in_f, (float*)ey->ptr,
                   (int)out_f, nullptr, GE_STORE, ws, wsbytes);
}

}  // extern "C"
