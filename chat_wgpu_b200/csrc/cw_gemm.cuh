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
// an f64 dot is ~1e-4 on the synthetic benchmark distribution, versus ~0.7 for
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
    int ksplit;           // K ranges per output tile (split-K for short M, few N tiles)
    float* ws;            // ksplit > 1: partial tiles [ksplit][M][N], summed by k_gemm_reduce
};

// Split-K workspaces: GM_WS_CTR words reserved at the start, then the partials.
constexpr int GM_WS_CTR = 2048;

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
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
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

// ---- operand preparation -------------------------------------------------------
// x -> (h, l) with x ~= h + l / 2^12: the f16 hi/lo pair the GEMM consumes.
__device__ __forceinline__ void split_f16(float x, __half* h, __half* l) {
    __half hh = __float2half_rn(x);
    *h = hh;
    *l = __float2half_rn((x - __half2float(hh)) * GM_LO);
}

}  // namespace cw
