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
    // setup above overlaps the previous kernel (PDL); inputs are read below
    pdl_trigger();
    pdl_wait();

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
    pdl_trigger();
    pdl_wait();
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
// Short-M product with the roles swapped: the 128 W rows of a tile are the
// MMA's M (operand A, dequantised into shared memory) and the M <= 256
// activation rows its N (operand B, NX = M rounded up to 16), so the tensor
// work is 128 x NX per K step instead of 128 x 128 -- at a decode batch of 8
// sessions 1/8 of it.  Two MMA stages (Wh, Wl 16 KB each, Xh, Xl NX*128 B
// each, 1024-byte aligned) and a deeper ring of raw records, so the weight
// stream from HBM runs ahead of the dequantisation.
constexpr int GQ_ST_MAX = 6, GQ_RS_MAX = 16;
// warp 0 X producer, warp 1 MMA issuer, warps 2-17 dequantise (4 threads per
// W row, two 8-weight chunks each; warps 2-5 also drain TMEM), warp 18 W producer
constexpr int GQ_CONV = 512;
constexpr int GQ_THREADS = 64 + GQ_CONV + 32;
constexpr int GQ_WPROD = (64 + GQ_CONV) / 32;
constexpr size_t GQ_SMEM_CAP = 226 * 1024;  // dynamic; the kernel also has static shared memory
constexpr size_t GQ_FIXED = 1024 + 512;  // alignment slack + barriers
__host__ __device__ constexpr int gq_stage_bytes(int nx) { return 2 * GM_TILE + 2 * nx * 128; }
// MMA stages: as many as fit next to an 8-deep raw ring (2..6) -- the MMA
// completion latency is hidden by the stages in flight, not by MMA work
__host__ __device__ constexpr int gq_stages(int nx) {
    return (int)((GQ_SMEM_CAP - GQ_FIXED - 8 * (size_t)GQ_REC) / gq_stage_bytes(nx)) > GQ_ST_MAX
               ? GQ_ST_MAX
           : (int)((GQ_SMEM_CAP - GQ_FIXED - 8 * (size_t)GQ_REC) / gq_stage_bytes(nx)) < 2
               ? 2
               : (int)((GQ_SMEM_CAP - GQ_FIXED - 8 * (size_t)GQ_REC) / gq_stage_bytes(nx));
}
__host__ __device__ constexpr int gq_ring(int nx) {  // raw ring depth that fits
    return (int)((GQ_SMEM_CAP - GQ_FIXED - (size_t)gq_stages(nx) * gq_stage_bytes(nx)) / GQ_REC) <
                   GQ_RS_MAX
               ? (int)((GQ_SMEM_CAP - GQ_FIXED - (size_t)gq_stages(nx) * gq_stage_bytes(nx)) /
                       GQ_REC)
               : GQ_RS_MAX;
}
__host__ __device__ constexpr size_t gq_smem(int nx) {
    return (size_t)gq_stages(nx) * gq_stage_bytes(nx) + (size_t)gq_ring(nx) * GQ_REC + GQ_FIXED;
}

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
// Half2 arithmetic, two weights per instruction: nibble n becomes the f16
// 1024 + n (exponent bits 0x6400 | n), minus 1032 gives q - 8 exactly;
// hi = f16(q*d) is one correctly rounded multiply of exact operands, and
// lo = f16(q*(d*2^12) - hi*2^12) one fused multiply-add of exact operands,
// i.e. the same pair as rounding (q-8)*d in f32 and its remainder.  Scales
// with |d| > 1 (where d*2^12 or hi*2^12 could overflow f16) take the f32 path.
__device__ __forceinline__ void gq_chunk_f32(const uint2 bytes8, bool high, float d, uint4* hi,
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

__device__ __forceinline__ __half2 u32_as_h2(uint32_t v) { return *reinterpret_cast<__half2*>(&v); }
__device__ __forceinline__ uint32_t h2_as_u32(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }

__device__ __forceinline__ void gq_chunk(const uint2 bytes8, bool high, float d, uint4* hi,
                                         uint4* lo) {
    if (!(fabsf(d) <= 1.0f)) {
        gq_chunk_f32(bytes8, high, d, hi, lo);
        return;
    }
    const __half2 d2 = __float2half2_rn(d);                 // exact: d came from an f16
    const __half2 D2 = __float2half2_rn(d * GM_LO);         // exact: power-of-two scaling
    const __half2 k12 = __float2half2_rn(GM_LO);
    const __half2 bias = u32_as_h2(0x64086408u);            // 1032 in both halves
    uint32_t ho[4], lo_[4];
#pragma unroll
    for (int w = 0; w < 2; w++) {
        const uint32_t v = (w ? bytes8.y : bytes8.x) >> (high ? 4 : 0);
        const __half2 q02 = __hsub2(u32_as_h2((v & 0x000f000fu) | 0x64006400u), bias);
        const __half2 q13 = __hsub2(u32_as_h2(((v >> 8) & 0x000f000fu) | 0x64006400u), bias);
        const __half2 h02 = __hmul2(q02, d2), h13 = __hmul2(q13, d2);
        const __half2 l02 = __hfma2(q02, D2, __hneg2(__hmul2(h02, k12)));
        const __half2 l13 = __hfma2(q13, D2, __hneg2(__hmul2(h13, k12)));
        const uint32_t a = h2_as_u32(h02), b = h2_as_u32(h13);
        const uint32_t c = h2_as_u32(l02), e = h2_as_u32(l13);
        ho[2 * w] = __byte_perm(a, b, 0x5410);      // weights 4w, 4w+1
        ho[2 * w + 1] = __byte_perm(a, b, 0x7632);  // weights 4w+2, 4w+3
        lo_[2 * w] = __byte_perm(c, e, 0x5410);
        lo_[2 * w + 1] = __byte_perm(c, e, 0x7632);
    }
    *hi = make_uint4(ho[0], ho[1], ho[2], ho[3]);
    *lo = make_uint4(lo_[0], lo_[1], lo_[2], lo_[3]);
}

// k_gemm_x3 with W read as packed Q4_0 records: warps 2-5 (one thread per W
// row) dequantise each stage's record into the swizzled f16 hi/lo tiles the
// MMA reads (the same values k_q4_split produces), then drain TMEM as the
// epilogue.  Streams 0.5625 bytes per weight instead of 4.
__global__ void __launch_bounds__(GQ_THREADS, 1)
    k_gemm_q4(const __grid_constant__ CUtensorMap tXh, const __grid_constant__ CUtensorMap tXl,
              const uint8_t* __restrict__ wpack, GemmArgs a, int nx) {
    extern __shared__ uint8_t gm_raw[];
    uint8_t* sm = (uint8_t*)(((uintptr_t)gm_raw + 1023) & ~(uintptr_t)1023);
    const int SB = gq_stage_bytes(nx), RS = gq_ring(nx), ST = gq_stages(nx);
    uint8_t* rings = sm + (size_t)ST * SB;                         // raw records
    uint64_t* full = (uint64_t*)(rings + (size_t)RS * GQ_REC);     // X tiles landed
    uint64_t* bfull = full + GQ_ST_MAX;                            // W tiles written
    uint64_t* empty = bfull + GQ_ST_MAX;                           // stage consumed by the MMAs
    uint64_t* rfull = empty + GQ_ST_MAX;                           // raw record landed
    uint64_t* rempty = rfull + GQ_RS_MAX;                          // raw record dequantised
    uint64_t* done = rempty + GQ_RS_MAX;
    uint32_t* tslot = (uint32_t*)(done + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nt = blockIdx.x / a.ksplit, ks = blockIdx.x % a.ksplit;
    const int n0 = nt * GM_BN;  // W rows of this tile
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
    // TMEM: two accumulators of nx columns, allocated as a power of two >= 32
    uint32_t cols = 32;
    while (cols < 2u * (uint32_t)nx) cols <<= 1;

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&bfull[s], GQ_CONV / 32);  // one arrival per converter warp
            mbar_init(&empty[s], 1);
        }
        for (int r = 0; r < RS; r++) {
            mbar_init(&rfull[r], 1);
            mbar_init(&rempty[r], GQ_CONV / 32);
        }
        mbar_init(done, 1);
        fence_mbar_init();
        tma_prefetch_desc(&tXh);
        tma_prefetch_desc(&tXl);
    }
    if (warp == 1) tmem_alloc(tslot, cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    // weight records are constant: start streaming them before the
    // dependency wait, which only the X tiles and the output need
    if (warp == GQ_WPROD) {
        if (lane == 0) {  // ---- W record producer
            int kb = 0;
            for (; kb < KB; kb++) {
                const int r = kb % RS;
                if (kb >= RS && !mbar_wait(&rempty[r], ((kb / RS) - 1) & 1, GM_WAIT_NS)) {
                    gm_fail(a.status);
                    break;
                }
                mbar_expect_tx(&rfull[r], GQ_REC);
                bulk_g2s(rings + (size_t)r * GQ_REC, wtile + (size_t)kb * GQ_REC, GQ_REC, &rfull[r]);
            }
            for (int j = max(0, kb - RS); j < kb; j++)
                if (!mbar_wait(&rfull[j % RS], (j / RS) & 1, GM_WAIT_NS)) gm_fail(a.status);
        }
    }
    pdl_trigger();
    pdl_wait();

    if (warp == 0) {
        if (lane == 0) {  // ---- X tile producer (TMA), nx rows per tile
            const unsigned xbytes = 2u * (unsigned)nx * GM_BK * 2u;
            int kb = 0;
            for (; kb < KB; kb++) {
                const int s = kb % ST;
                if (kb >= ST && !mbar_wait(&empty[s], ((kb / ST) - 1) & 1, GM_WAIT_NS)) {
                    gm_fail(a.status);
                    break;
                }
                uint8_t* st = sm + (size_t)s * SB + 2 * GM_TILE;
                mbar_expect_tx(&full[s], xbytes);
                const int kx = (kb0 + kb) * GM_BK;
                tma_load_2d(st, &tXh, kx, 0, &full[s]);
                tma_load_2d(st + nx * 128, &tXl, kx, 0, &full[s]);
            }
            for (int j = max(0, kb - ST); j < kb; j++)
                if (!mbar_wait(&full[j % ST], (j / ST) & 1, GM_WAIT_NS)) gm_fail(a.status);
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer: D[W rows][x rows] += W . X^T
            const uint32_t idesc = umma_idesc_f16(GM_BN, nx);
            const uint32_t acc_hi = tmem, acc_lo = tmem + (uint32_t)nx;
            for (int kb = 0; kb < KB; kb++) {
                const int s = kb % ST;
                if (!mbar_wait(&full[s], (kb / ST) & 1, GM_WAIT_NS) ||
                    !mbar_wait(&bfull[s], (kb / ST) & 1, GM_WAIT_NS)) {
                    gm_fail(a.status);
                    break;
                }
                tc_fence_after();
                const uint32_t st = smem_addr(sm + (size_t)s * SB);
                const uint64_t dwh = umma_desc_sw128(st), dwl = umma_desc_sw128(st + GM_TILE);
                const uint64_t dxh = umma_desc_sw128(st + 2 * GM_TILE),
                               dxl = umma_desc_sw128(st + 2 * GM_TILE + nx * 128);
#pragma unroll
                for (int k = 0; k < GM_BK / 16; k++) {
                    const uint64_t adv = (uint64_t)(k * 32) >> 4;
                    const uint32_t first = (kb > 0 || k > 0) ? 1u : 0u;
                    umma_f16(acc_hi, dwh + adv, dxh + adv, idesc, first);
                    umma_f16(acc_lo, dwh + adv, dxl + adv, idesc, first);
                    umma_f16(acc_lo, dwl + adv, dxh + adv, idesc, 1u);
                }
                tc_commit(&empty[s]);
            }
            tc_commit(done);
        }
    } else if (warp < GQ_WPROD) {  // ---- warps 2..17: dequantise W records; 2..5: epilogue
        const int t = threadIdx.x - 64;
        const int row = t & (GM_BN - 1), part = t >> 7;  // W row, chunk pair 2part, 2part+1
        bool ok = true;
        for (int kb = 0; kb < KB && ok; kb++) {
            const int s = kb % ST, r = kb % RS;
            // the raw record has landed and the MMAs are done with this stage's W tiles
            if (!mbar_wait(&rfull[r], (kb / RS) & 1, GM_WAIT_NS) ||
                (kb >= ST && !mbar_wait(&empty[s], ((kb / ST) - 1) & 1, GM_WAIT_NS))) {
                gm_fail(a.status);
                ok = false;
                break;
            }
            uint8_t* st = sm + (size_t)s * SB;
            const uint8_t* rec = rings + (size_t)r * GQ_REC;
            const uint4 pay = *(const uint4*)(rec + row * 32 + (part >> 1) * 16);
            const __half2 sc = *(const __half2*)(rec + GM_BN * 32 + row * 4);
            __syncwarp();  // the warp's record reads are done: one arrival frees the slot
            if (lane == 0) mbar_arrive(&rempty[r]);
            const float d = (part >> 1) ? __high2float(sc) : __low2float(sc);
            uint8_t* wh = st + row * 128;
            uint8_t* wl = st + GM_TILE + row * 128;
            const int sw = row & 7;
            const bool high = part & 1;  // chunks 2, 3 of a block: high nibbles
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int c = 2 * part + u;
                const uint2 b8 = u ? make_uint2(pay.z, pay.w) : make_uint2(pay.x, pay.y);
                uint4 h, l;
                gq_chunk(b8, high, d, &h, &l);
                *(uint4*)(wh + ((c ^ sw) << 4)) = h;
                *(uint4*)(wl + ((c ^ sw) << 4)) = l;
            }
            fence_proxy_async();  // generic-proxy stores -> visible to the MMA's async proxy
            __syncwarp();
            if (lane == 0) mbar_arrive(&bfull[s]);  // per warp: 512 thread arrivals serialise
        }
        if (warp > 5) goto gq_end;
        const bool ok_done = mbar_wait(done, 0, GM_WAIT_NS);
        if (!ok_done) gm_fail(a.status);
        ok = ok && ok_done;
        tc_fence_after();
        // TMEM lane = W row n, column = activation row m
        const int q = warp & 3;
        const int n = n0 + q * 32 + lane;
        const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
        const float bn = (bias && n < a.N) ? bias[n] : 0.f;
#pragma unroll 1
        for (int c = 0; c < nx; c += 16) {
            uint32_t h[16], l[16];
            tmem_ld16(lane_base + c, h);
            tmem_ld16(lane_base + nx + c, l);
            tmem_wait_ld();
            if (!ok || n >= a.N) continue;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int m = c + j;
                if (m >= a.M) break;
                float v = __uint_as_float(h[j]) + __uint_as_float(l[j]) * (1.0f / GM_LO) + bn;
                float* dst = ybase + (size_t)m * ldy + n;
                if (epi == GE_ADD) v += *dst;
                *dst = v;
            }
        }
    }
gq_end:
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, cols);
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
static int tmap_f16(CUtensorMap* map, const void* base, long rows, int K, int box_rows = GM_BM) {
    auto enc = tmap_encode_fn();
    CW_CHECK(enc, CW_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    CW_CHECK(((uintptr_t)base & 15) == 0 && K % 8 == 0, CW_ERR_INVALID_ARG,
             "gemm operand must be 16-byte aligned with K %% 8 == 0");
    cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {(cuuint32_t)GM_BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides,
                     box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    CW_CHECK(r == CUDA_SUCCESS, CW_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return CW_OK;
}

int gemm_x3(cw_ctx* ctx, const void* xh, const void* xl, const void* wh, const void* wl, int M,
            int N, int K, float* y, int ldy, const float* bias, int epi, float* ws,
            size_t ws_bytes, bool pdl) {
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
               (size_t)(ks * 2) * M * N * 4 + GM_WS_CTR * 4 <= ws_bytes)
            ks *= 2;
    {  // every split gets at least one K step
        const int per = (KB + ks - 1) / ks;
        ks = (KB + per - 1) / per;
    }
    a.ksplit = ks;
    a.ws = ws ? ws + GM_WS_CTR : nullptr;  // workspace layout shared with k_gemm_q4
    CW_TRY(launch_pdl(ctx, pdl, k_gemm_x3, dim3(m_tiles * n_tiles * ks), dim3(192), GM_SMEM,
                      m_xh, m_xl, m_wh, m_wl, a));
    CW_TRY(check_launch("gemm_x3"));
    if (ks == 1) return CW_OK;
    const long n = (long)M * N;
    const int grid = (int)std::min<long>((n + 255) / 256, (long)ctx->sm_count * 8);
    CW_TRY(launch_pdl(ctx, pdl, k_gemm_reduce, dim3(grid), dim3(256), 0, (const float*)a.ws, ks,
                      M, N, y, ldy, bias, epi));
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
            float* y, int ldy, const float* bias, int epi, float* ws, size_t ws_bytes, bool pdl) {
    CW_CHECK(M > 0 && N > 0 && K > 0 && K % 32 == 0 && ldy >= N, CW_ERR_INVALID_ARG,
             "gemm: bad shape M=%d N=%d K=%d ldy=%d", M, N, K, ldy);
    CW_CHECK(((uintptr_t)wpack & 15) == 0, CW_ERR_INVALID_ARG, "gemm: packed W not 16-byte aligned");
    CW_CHECK(M <= 256, CW_ERR_INVALID_ARG, "gemm_q4: M=%d above the 256 rows of one tile", M);
    // the activation rows are the MMA's N: a multiple of 16 (M = 128 shape)
    const int nx = (M + 15) / 16 * 16;
    CUtensorMap m_xh, m_xl;
    CW_TRY(tmap_f16(&m_xh, xh, M, K, nx));
    CW_TRY(tmap_f16(&m_xl, xl, M, K, nx));
    static bool attr_set[64] = {};
    if (!attr_set[ctx->device & 63]) {
        CW_CUDA(cudaFuncSetAttribute(k_gemm_q4, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)GQ_SMEM_CAP));
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
    const int n_tiles = (N + GM_BN - 1) / GM_BN;
    const int KB = (K + GM_BK - 1) / GM_BK;
    int ks = 1;
    if (ws)
        while (n_tiles <= GM_WS_CTR && n_tiles * ks * 2 < 2 * ctx->sm_count &&
               ks * 2 <= KB / 2 && ks < 32 &&
               (size_t)(ks * 2) * M * N * 4 + GM_WS_CTR * 4 <= ws_bytes)
            ks *= 2;
    {  // every split gets at least one K step
        const int per = (KB + ks - 1) / ks;
        ks = (KB + per - 1) / per;
    }
    a.ksplit = ks;
    a.ws = ws ? ws + GM_WS_CTR : nullptr;
    CW_TRY(launch_pdl(ctx, pdl, k_gemm_q4, dim3(n_tiles * ks), dim3(GQ_THREADS), gq_smem(nx),
                      m_xh, m_xl, (const uint8_t*)wpack, a, nx));
    CW_TRY(check_launch("gemm_q4"));
    if (ks == 1) return CW_OK;
    // partial tiles summed in split order (deterministic) by a grid over all of
    // Y: an in-kernel "last CTA reduces" pass serialises M x ksplit loads per thread
    const long n = (long)M * N;
    const int grid = (int)std::min<long>((n + 255) / 256, (long)ctx->sm_count * 8);
    CW_TRY(launch_pdl(ctx, pdl, k_gemm_reduce, dim3(grid), dim3(256), 0, (const float*)a.ws, ks,
                      M, N, y, ldy, bias, epi));
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
        CW_CUDA(cudaMemsetAsync(ctx->gemm_scratch, 0, bytes, ctx->stream));  // split-K counters
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
    // the split-K workspace (with its self-resetting counters) sits at a fixed
    // place, the start of the scratch
    const size_t wsbytes = 32ull << 20;
    uint8_t* sc = nullptr;
    CW_TRY(gemm_scratch(ctx, wsbytes + 2 * xbytes + wbytes, &sc));
    float* ws = (float*)sc;
    uint8_t *xh = sc + wsbytes, *xl = xh + xbytes, *wp = xl + xbytes;
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
