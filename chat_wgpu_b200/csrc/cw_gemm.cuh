// cw_gemm.cuh -- the prefill Q4_0 GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM, operands staged by TMA).
//
//   Y[M, N] = X[M, K] . W[N, K]^T      W packed GGUF Q4_0, X f32
//
// The reference has no batched prefill: its prompt runs token by token
// through q4.wgsl's f32 dequant-dot (src/model/mod.rs:78-83,
// src/kernels/q4.wgsl:40-73).  To stay within that path's 1e-3 relative
// tolerance on tensor cores, both operands are split into two f16 terms:
//
//   W = Wh + Wl / 2^12   Wh = f16(W), Wl = f16((W - Wh) * 2^12)   (exact: a
//                        Q4_0 weight (q-8)*d has at most 14 significant bits)
//   X = Xh + Xl / 2^12   Xh = f16(X), Xl = f16((X - Xh) * 2^12)   (22 bits)
//
//   Y = Xh.Wh  +  (Xh.Wl + Xl.Wh) / 2^12        (the Xl.Wl term is below 2^-22)
//
// Three MMAs per K step into two f32 TMEM accumulators; the scaled low terms
// keep every f16 operand in the normal range.  Max relative error against
// an f64 dot is ~1e-4 on the SURVEY synthetic distribution, versus ~0.7 for
// a single f16 pass (measured with the 1e-3*rms floor of the parity rule).
//
// Tile: 128 (M, one TMEM lane per row) x 128 (N) x 64 (K, one 128-byte
// swizzle atom of f16), 3 stages of four 16 KB tiles in shared memory.
// Warp roles (192 threads): warp 0 lane 0 issues the TMA loads, warp 1
// allocates TMEM and lane 0 issues the MMAs, warps 2-5 drain the
// accumulators (a warp reaches TMEM lanes 32*(warp%4) .. +31).
// Every mbarrier wait is bounded; a timeout sets the device status word and
// the kernel still frees its TMEM.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "cw_gemv.cuh"  // mbarrier / smem helpers

namespace cw {

constexpr int GM_BM = 128, GM_BN = 128, GM_BK = 64, GM_ST = 3;
constexpr int GM_TILE = GM_BM * GM_BK * 2;              // bytes of one f16 operand tile
constexpr int GM_STAGE = 4 * GM_TILE;                   // Xh, Xl, Wh, Wl
constexpr int GM_TMEM_COLS = 2 * GM_BN;                 // hi and lo accumulators
constexpr size_t GM_SMEM = (size_t)GM_ST * GM_STAGE + 256 + 1024;  // + barriers, align slack
constexpr float GM_LO = 4096.f;                         // scale of the low terms
constexpr uint64_t GM_WAIT_NS = 2000000000ull;

enum GemmEpi : int { GE_STORE = 0, GE_ADD = 1 };

struct GemmArgs {
    float* y;             // [M, ldy]
    const float* bias;    // [N] or null
    int M, N, K, ldy;
    int epi;              // GE_STORE: y = acc (+bias); GE_ADD: y += acc (+bias)
    int group_m;          // M tiles per raster group (L2 reuse of W tiles)
    int* status;          // device status word
};

// ---- tcgen05 / TMA primitives ---------------------------------------------------
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_addr(slot)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
                 : "memory");
}
// Shared-memory matrix descriptor: K-major operand in the canonical 128-byte
// swizzled layout (8-row groups 1024 bytes apart), descriptor version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16)  // LBO (unused when swizzled)
           | ((uint64_t)(1024 >> 4) << 32)                            // SBO
           | ((uint64_t)1 << 46)                                      // version
           | ((uint64_t)2 << 61);                                     // SWIZZLE_128B
}
// Instruction descriptor, kind::f16: f16 x f16 -> f32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
    return (1u << 4)                    // D f32
           | (0u << 7) | (0u << 10)     // A, B f16
           | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once every tcgen05 operation this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 2-D tiled TMA load (no multicast); x is the inner (K) coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_addr(dst)),
        "l"((uint64_t)map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

__device__ __forceinline__ void gm_fail(int* status) {
    if (status) atomicCAS(status, DEV_OK, DEV_TIMEOUT);
}

// Tile (m, n) of linear block id `bid` with M tiles grouped `group_m` at a
// time, so the CTAs resident together share W tiles through L2.
__device__ __forceinline__ void gm_tile(int bid, int m_tiles, int n_tiles, int group_m, int* mt,
                                        int* nt) {
    const int per_group = group_m * n_tiles;
    const int g = bid / per_group;
    const int first = g * group_m;
    const int gsize = min(m_tiles - first, group_m);
    const int r = bid - g * per_group;
    *mt = first + r % gsize;
    *nt = r / gsize;
}

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
    gm_tile(blockIdx.x, m_tiles, n_tiles, a.group_m, &mt, &nt);
    const int m0 = mt * GM_BM, n0 = nt * GM_BN;
    const int KB = (a.K + GM_BK - 1) / GM_BK;

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
                const int kx = kb * GM_BK;
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
            float* yr = a.y + (size_t)row * a.ldy;
            const int nb = n0 + c;
            if (nb + 16 <= a.N && (a.ldy & 3) == 0) {
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                    float r[4];
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        r[t] = __uint_as_float(h[j + t]) +
                               __uint_as_float(l[j + t]) * (1.0f / GM_LO);
                        if (a.bias) r[t] += a.bias[nb + j + t];
                    }
                    float4* dst = (float4*)(yr + nb + j);
                    if (a.epi == GE_ADD) {
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
                    if (a.bias) acc += a.bias[nb + j];
                    if (a.epi == GE_ADD) acc += yr[nb + j];
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

// ---- operand preparation ----------------------------------------------------------
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

__device__ __forceinline__ void split_f16(float x, __half* h, __half* l) {
    __half hh = __float2half_rn(x);
    *h = hh;
    *l = __float2half_rn((x - __half2float(hh)) * GM_LO);
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

}  // namespace cw
