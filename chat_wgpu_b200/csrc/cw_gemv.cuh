// cw_gemv.cuh -- the streaming Q4 GEMV: y[N] = W[N,K] x for Q4 weights,
// shared by the stand-alone op entry points and the fused decode kernels.
// The same kernel streams GGUF Q4_K / Q5_K super-blocks and the aligned
// Q6_K split (layouts in cw_device.cuh; per-unit math in kq_chunk).
//
// Data movement (B200): weight rows are contiguous in both planes (16-byte
// nibble payloads, then f16/f32 scales), so a CTA streams "chunks" of RC
// consecutive rows with two cp.async.bulk copies per chunk into a ring of S
// shared-memory stages, completion tracked by one mbarrier per stage.  One
// elected thread issues the copies; the first S chunks are issued before
// griddepcontrol.wait, i.e. while the previous kernel of the decode step is
// still running.  A chunk is 8-16 KB, so each SM keeps up to ~140 KB of
// weights in flight with two CTAs resident.
//
// Arithmetic: x is converted once per CTA to q24 block-floating-point planes
// (cw_device.cuh) and each lane keeps the planes of its BPL blocks in
// registers for the whole kernel; a weight block then costs one shared-memory
// load, 12 bit ops, 24 dp4a and a few flops.
//
// Work mapping: 8 warps; WPR warps share a row (lanes over its blocks,
// block b = (warp % WPR)*32 + lane + k*32*WPR, k < BPL), 8/WPR row slots per
// chunk, RPW rows per slot: RC = (8/WPR)*RPW rows per chunk.  Per-row sums go
// through shared memory and are added in a fixed order, so results are
// bit-reproducible run to run.
//
// Waits are bounded by %globaltimer: a wait that exceeds the limit records
// DEV_TIMEOUT in the status word, waits (bounded) for the copies in flight
// and ends the kernel; the host reports CW_ERR_TIMEOUT.
#pragma once

#include <stdint.h>

#include "cw_common.h"
#include "cw_device.cuh"

namespace cw {

enum { PRO_X = 0, PRO_NORM = 1 };
enum { EPI_STORE = 0, EPI_RESID = 1, EPI_GLU = 2, EPI_HEAD = 3 };

struct GemvArgs {
    const uint8_t* payload;  // [N][K/32][16]
    const void* scales;      // [N][K/32] f16 (GGUF) or f32 (crate layout)
    int K, N;
    // PRO_X: x [K] from global memory
    const float* x;
    // PRO_NORM: h = base (+ delta, post-normed with post_w when non-null);
    // x = rmsnorm(h) * gain(norm_w); h written to h_out and x to xn_out by CTA 0
    const float* base;
    int base_smem;  // base points to this CTA's shared memory
    const float* delta;
    const float* post_w;
    float* h_out;
    const float* norm_w;
    float* xn_out;
    float eps;
    int unit;  // UnitShift gain (1 + w)
    // epilogue
    float* y;
    const float* bias;              // EPI_STORE: optional per-row bias
    int geglu;                      // EPI_GLU: 0 SwiGLU, 1 GeGLU (rows 2i = gate_i, 2i+1 = up_i)
    float softcap;                  // EPI_HEAD: tanh soft-cap of the logits (0 = off)
    unsigned key_offset;            // EPI_HEAD: index of row 0 in the full vocabulary (TP shard)
    unsigned long long* key;        // EPI_HEAD: argmax accumulator (atomicMax)
    int* status;                    // device status word
};

template <int WPR_, int BPL_, int RPW_>
struct GemvCfg {
    static constexpr int WPR = WPR_, BPL = BPL_, RPW = RPW_;
    static constexpr int SLOTS = 8 / WPR;
    static constexpr int RC = SLOTS * RPW;
    static constexpr int NB_MAX = 32 * WPR * BPL;
};
using GemvC32 = GemvCfg<1, 1, 4>;   // K <= 1024:  32 rows per chunk
using GemvC64 = GemvCfg<1, 2, 2>;   // K <= 2048:  16 rows
using GemvC96 = GemvCfg<1, 3, 2>;   // K <= 3072:  16 rows
using GemvC128 = GemvCfg<2, 2, 2>;  // K <= 4096:   8 rows (18 KB chunks at 4096, no idle lanes)
using GemvC192 = GemvCfg<2, 3, 2>;  // K <= 6144:   8 rows
using GemvC256 = GemvCfg<4, 2, 2>;  // K <= 8192:   4 rows
using GemvC384 = GemvCfg<4, 3, 2>;  // K <= 12288:  4 rows
using GemvC768 = GemvCfg<8, 3, 1>;  // K <= 24576:  1 row

constexpr uint64_t GEMV_WAIT_NS = 2000000000ull;  // 2 s

// ---- mbarrier / bulk-copy helpers ----------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for the phase with `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity))
        if (global_ns() - t0 > limit_ns) return false;
    return true;
}
// Global -> this CTA's shared memory, completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// Same copy with an L2 cache-policy hint (see l2_evict_first).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, unsigned bytes,
                                              uint64_t* bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
// L2 policy for data read once per step (the weight stream): its lines are
// the first to go, so the KV cache, activations and small parameters stay
// resident in L2 while hundreds of MB of weights pass through.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__host__ __device__ constexpr size_t al128(size_t v) { return (v + 127) / 128 * 128; }
__host__ __device__ constexpr size_t al16(size_t v) { return (v + 15) / 16 * 16; }

// Bytes per 32-weight unit in the weight stream: the payload plane (Q4_0
// nibbles; the k-quants' whole super-blocks, headers included) and the
// separate scale plane (f16 / f32 for Q4_0, none for the k-quants).
template <int LAYOUT>
__host__ __device__ constexpr int gemv_pbb() {
    return LAYOUT == LAYOUT_Q4K ? 18 : LAYOUT == LAYOUT_Q5K ? 22 : LAYOUT == LAYOUT_Q6K ? 26
         : LAYOUT == LAYOUT_Q8  ? 32 : 16;
}
template <int LAYOUT>
__host__ __device__ constexpr int gemv_sw() {
    return (LAYOUT == LAYOUT_GGUF || LAYOUT == LAYOUT_Q8) ? 2 : LAYOUT == LAYOUT_REF ? 4 : 0;
}
// Scale-plane bytes of `rows` rows and their offset in the plane: Q6_K's f16
// d per super-block, its copy rounded up to 16 bytes (the plane's buffer is
// padded to 256 bytes, so the rounded copy stays inside it).
template <int LAYOUT>
__host__ __device__ constexpr size_t gemv_sc_bytes(long rows, int nb) {
    return LAYOUT == LAYOUT_Q6K ? al16((size_t)rows * (nb / 8) * 2)
                                : (size_t)rows * nb * gemv_sw<LAYOUT>();
}
template <int LAYOUT>
__host__ __device__ constexpr size_t gemv_sc_off(long row0, int nb) {
    return LAYOUT == LAYOUT_Q6K ? (size_t)row0 * (nb / 8) * 2 : (size_t)row0 * nb * gemv_sw<LAYOUT>();
}

// Shared-memory layout sizes (bytes).
struct GemvSmem {
    size_t pay, sc, stage, q24, hbuf, red, total;
    __host__ __device__ GemvSmem(int RC, int WPR, int nb, int pbb, size_t scb, int S, int K,
                                 bool norm) {
        pay = al128((size_t)RC * nb * pbb);
        sc = al128(scb);
        stage = pay + sc;
        q24 = al16(q24_bytes(nb));
        hbuf = norm ? al16((size_t)K * 4) : 0;
        red = al16((size_t)2 * RC * WPR * 4);
        total = 128 + (size_t)S * stage + q24 + hbuf + red;
    }
};

// Sum over the CTA (up to 32 warps); red holds one float per warp.
__device__ __forceinline__ float gemv_cta_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

// Reduce RPW (1, 2 or 4) per-lane partials across the warp in 5 shuffles:
// the first log2(RPW) butterfly steps exchange whole rows instead of summing
// them, so afterwards lanes [j*32/RPW, (j+1)*32/RPW) hold row j's total.
// The order of additions is fixed, so the result is reproducible.
template <int RPW>
__device__ __forceinline__ float warp_reduce_rows(const float (&v)[RPW], int lane) {
    if constexpr (RPW == 1) {
        return warp_sum(v[0]);
    } else if constexpr (RPW == 2) {
        const bool up = lane & 16;
        float keep = up ? v[1] : v[0];
        const float send = up ? v[0] : v[1];
        keep += __shfl_xor_sync(FULL, send, 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(FULL, keep, o);
        return keep;
    } else {
        static_assert(RPW == 4, "rows per warp must be 1, 2 or 4");
        const bool up = lane & 16;
        float k0 = up ? v[2] : v[0], k1 = up ? v[3] : v[1];
        const float s0 = up ? v[0] : v[2], s1 = up ? v[1] : v[3];
        k0 += __shfl_xor_sync(FULL, s0, 16);
        k1 += __shfl_xor_sync(FULL, s1, 16);
        const bool up2 = lane & 8;
        float k = up2 ? k1 : k0;
        const float s = up2 ? k0 : k1;
        k += __shfl_xor_sync(FULL, s, 8);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) k += __shfl_xor_sync(FULL, k, o);
        return k;
    }
}

__device__ __forceinline__ float silu_ref_f(float x) { return x / (1.0f + expf(-x)); }  // glu.wgsl:25
__device__ __forceinline__ float gelu_ref_f(float x) {                                 // glu.wgsl:27-30
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

constexpr int GEMV_PB = 8;  // residual elements per thread per load batch

// x -> q24 planes in shared memory (PRO_X: x from global; PRO_NORM: the
// rmsnorm prologue of the decode kernels, norm.wgsl:20-56).
template <int LAYOUT, int PRO>
__device__ __forceinline__ void gemv_prologue(const GemvArgs& a, const Q24& q, float* hbuf,
                                              float* red8) {
    const int nb = a.K / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = blockDim.x >> 5, sub = lane >> 3, e0 = 4 * (lane & 7);
    if (PRO == PRO_X) {
        if constexpr (LAYOUT != LAYOUT_REF) {  // four elements per lane (q24_quad); nb % 8 == 0
            for (int t = warp; t < nb / 4; t += nw) {
                const int b = 4 * t + sub;
                q24_quad(q, b, true,
                         __ldcg(reinterpret_cast<const float4*>(a.x + unit_elem<LAYOUT>(b, e0))),
                         lane);
            }
        } else {
            for (int b = warp; b < nb; b += nw) q24_block<LAYOUT>(q, b, __ldcg(a.x + b * 32 + lane), lane);
        }
        return;
    }
    // base/delta may have been written by other CTAs of a persistent kernel:
    // read them through L2 (ld.global.cg), never from a stale L1 line
    // Each thread takes elements i = tid + u*blockDim.x in increasing order,
    // GEMV_PB of them per batch with every load of the batch issued before
    // the math (one L2 round trip per batch, not per element).
    const int K = a.K;
    float inv_d = 0.f;
    if (a.delta && a.post_w) {
        float ss = 0.f;
        for (int i0 = threadIdx.x; i0 < K; i0 += GEMV_PB * blockDim.x) {
            float dv[GEMV_PB];
#pragma unroll
            for (int u = 0; u < GEMV_PB; u++) {
                const int i = i0 + u * blockDim.x;
                dv[u] = i < K ? __ldcg(a.delta + i) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < GEMV_PB; u++)
                if (i0 + u * (int)blockDim.x < K) ss = fmaf(dv[u], dv[u], ss);
        }
        ss = gemv_cta_sum(ss, red8);
        inv_d = 1.0f / sqrtf(ss / (float)K + a.eps);
    }
    float ssh = 0.f;
    const bool wr = a.h_out && blockIdx.x == 0;
    for (int i0 = threadIdx.x; i0 < K; i0 += GEMV_PB * blockDim.x) {
        float hv[GEMV_PB], dv[GEMV_PB], gv[GEMV_PB];
#pragma unroll
        for (int u = 0; u < GEMV_PB; u++) {
            const int i = i0 + u * blockDim.x;
            const bool in = i < K;
            hv[u] = !in ? 0.f : a.base_smem ? a.base[i] : __ldcg(a.base + i);
            dv[u] = in && a.delta ? __ldcg(a.delta + i) : 0.f;
            gv[u] = in && a.delta && a.post_w ? a.post_w[i] : 0.f;
        }
#pragma unroll
        for (int u = 0; u < GEMV_PB; u++) {
            const int i = i0 + u * blockDim.x;
            if (i >= K) continue;
            float h = hv[u];
            if (a.delta) {
                float d = dv[u];
                if (a.post_w) {
                    const float gw = a.unit ? 1.0f + gv[u] : gv[u];
                    d = __fmul_rn(__fmul_rn(d, inv_d), gw);
                }
                h = h + d;
            }
            hbuf[i] = h;
            if (wr) a.h_out[i] = h;
            ssh = fmaf(h, h, ssh);
        }
    }
    ssh = gemv_cta_sum(ssh, red8);
    const float inv = 1.0f / sqrtf(ssh / (float)K + a.eps);
    const bool wx = a.xn_out && blockIdx.x == 0;
    if constexpr (LAYOUT != LAYOUT_REF) {  // four elements per lane (q24_quad); nb % 8 == 0
        for (int t = warp; t < nb / 4; t += nw) {
            const int b = 4 * t + sub, i = unit_elem<LAYOUT>(b, e0);
            const float4 h = *reinterpret_cast<const float4*>(hbuf + i);
            float4 g = __ldg(reinterpret_cast<const float4*>(a.norm_w + i));
            if (a.unit) g = make_float4(1.0f + g.x, 1.0f + g.y, 1.0f + g.z, 1.0f + g.w);
            const float4 v = make_float4(__fmul_rn(__fmul_rn(h.x, inv), g.x),
                                         __fmul_rn(__fmul_rn(h.y, inv), g.y),
                                         __fmul_rn(__fmul_rn(h.z, inv), g.z),
                                         __fmul_rn(__fmul_rn(h.w, inv), g.w));
            if (wx) *reinterpret_cast<float4*>(a.xn_out + i) = v;
            q24_quad(q, b, true, v, lane);
        }
    } else {
    for (int b = warp; b < nb; b += nw) {
        const int i = b * 32 + lane;
        const float gw = a.unit ? 1.0f + a.norm_w[i] : a.norm_w[i];
        const float v = __fmul_rn(__fmul_rn(hbuf[i], inv), gw);
        if (wx) a.xn_out[i] = v;
        q24_block<LAYOUT>(q, b, v, lane);
    }
    }
}

// The (scale, min) pairs of sub-blocks 2c and 2c+1 of a Q4_K / Q5_K
// super-block whose 16-byte header is h (.x = f16 d | f16 dmin << 16, .y .z .w
// = the 12 packed 6-bit scale/min bytes q[0..11]): for j < 4 scale q[j] & 63,
// min q[j+4] & 63; for j >= 4 scale (q[j+4] & 15) | (q[j-4] >> 6) << 4, min
// (q[j+4] >> 4) | (q[j] >> 6) << 4.  Both sub-blocks at once, one per byte
// of a 16-bit field.  Returns d*scale and dmin*min (exact in f32).
__device__ __forceinline__ void kq_scales(const uint4& h, int c, float& alo, float& ahi,
                                          float& blo, float& bhi) {
    // c is fixed per lane: the pair's masks are selects, not a branch
    const int sh = 16 * (c & 1);
    const bool big = c >= 2;
    const unsigned lowm = big ? 0x0f0fu : 0x3f3fu, hm = big ? 0x3030u : 0u;
    const unsigned y2 = h.y >> sh, z2 = h.z >> sh;
    const unsigned a2 = (big ? h.w : h.y) >> sh;
    const unsigned scp = (a2 & lowm) | ((y2 >> 2) & hm);
    const unsigned mp = ((big ? a2 >> 4 : z2) & lowm) | ((z2 >> 2) & hm);
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xffffu)));
    const float dm = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    // x (0..63) as the float 2^23 + x made from its bits, and d * x as
    // fma(d, 2^23 + x, -d * 2^23): one rounding of the exact d * x, which
    // has at most 17 significant bits, so the product is exact as before
    const float nd = -8388608.0f * d, ndm = -8388608.0f * dm;
    alo = fmaf(d, __uint_as_float(0x4B000000u | (scp & 0xffu)), nd);
    ahi = fmaf(d, __uint_as_float(0x4B000000u | ((scp >> 8) & 0xffu)), nd);
    blo = fmaf(dm, __uint_as_float(0x4B000000u | (mp & 0xffu)), ndm);
    bhi = fmaf(dm, __uint_as_float(0x4B000000u | ((mp >> 8) & 0xffu)), ndm);
}

// One stage of the k-quant GEMV: this warp's RPW rows x BPL units of the
// raw super-blocks in shared memory (pay: the chunk's rows back to back).
// Per unit, the low and high nibbles (+ Q5_K's fifth bits) are dotted with
// the unit's q24 planes apart (their sub-blocks have their own scales):
// sum = sb * (d*sc_lo * T_lo + d*sc_hi * T_hi) - (dmin*m_lo * sx_lo + dmin*m_hi * sx_hi)
// with T = D0 + 256 D1 + 65536 D2 the integer dot products of the planes.
//
// Q6_K: q = the nibble | two bits of qh << 4 (0..63), w = d * sc * (q - 32):
// sum = d * (sc_lo * (sb * T_lo - 32 sx_lo) + sc_hi * (sb * T_hi - 32 sx_hi)),
// the int8 scales and the f16 d from their planes (scs: the chunk's d values).
template <int LAYOUT, int RPW, int BPL, int WPR>
__device__ __forceinline__ void kq_chunk(const unsigned char* pay, const unsigned char* scs, int nb,
                                         int rows, int slot, int wsub, int lane, int c,
                                         const uint4 (&xa)[BPL][3], const uint4 (&xb)[BPL][3],
                                         const float (&sbr)[BPL], const float (&xsl)[BPL],
                                         const float (&xsh)[BPL], float (&acc)[RPW]) {
    constexpr bool FIVE = LAYOUT == LAYOUT_Q5K, SIX = LAYOUT == LAYOUT_Q6K;
    constexpr int SBB = SIX ? 208 : FIVE ? 176 : 144, QOFF = SIX ? 0 : FIVE ? 48 : 16;
    const int nbk = nb >> 3;
    // Q6_K: this lane's unit u = lane % 8 of each super-block (half u/4,
    // s = (u/2)%2, t = u%2): qh run 128 + 32h + 16t, scales 8h + 2s + t and + 4
    const int u6 = lane & 7, qh6 = 128 + 32 * (u6 >> 2) + 16 * (u6 & 1), sc6 = 192 + 8 * (u6 >> 2);
    const int sh6 = 2 * ((u6 >> 1) & 1), by6 = 8 * (u6 & 3);
    uint4 w4[RPW][BPL], h4[RPW][BPL], q5[RPW][(FIVE || SIX) ? BPL : 1];
    float d6[RPW][SIX ? BPL : 1];
#pragma unroll
    for (int j = 0; j < RPW; j++) {
        const int r = slot * RPW + j;
#pragma unroll
        for (int k = 0; k < BPL; k++) {
            const int b = wsub * 32 + lane + k * 32 * WPR;
            const bool in = r < rows && b < nb;
            const size_t sbi = (size_t)(in ? r : 0) * nbk + (in ? b >> 3 : 0);
            const unsigned char* sb = pay + sbi * SBB;
            const uint4 z = make_uint4(0, 0, 0, 0);
            w4[j][k] = in ? *reinterpret_cast<const uint4*>(sb + QOFF + (b & 7) * 16) : z;
            if constexpr (SIX) {
                q5[j][k] = in ? *reinterpret_cast<const uint4*>(sb + qh6) : z;
                const uint2 sc2 = in ? *reinterpret_cast<const uint2*>(sb + sc6) : make_uint2(0, 0);
                h4[j][k] = make_uint4(sc2.x, sc2.y, 0, 0);
                d6[j][k] = in ? __half2float(reinterpret_cast<const __half*>(scs)[sbi]) : 0.f;
            } else {
                h4[j][k] = in ? *reinterpret_cast<const uint4*>(sb) : z;
                if constexpr (FIVE)
                    q5[j][k] = in ? *reinterpret_cast<const uint4*>(sb + 16 + (b & 1) * 16) : z;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < RPW; j++) {
        acc[j] = 0.f;
#pragma unroll
        for (int k = 0; k < BPL; k++) {
            const unsigned w[4] = {w4[j][k].x, w4[j][k].y, w4[j][k].z, w4[j][k].w};
            const unsigned a0[4] = {xa[k][0].x, xa[k][0].y, xa[k][0].z, xa[k][0].w};
            const unsigned b0[4] = {xb[k][0].x, xb[k][0].y, xb[k][0].z, xb[k][0].w};
            const unsigned a1[4] = {xa[k][1].x, xa[k][1].y, xa[k][1].z, xa[k][1].w};
            const unsigned b1[4] = {xb[k][1].x, xb[k][1].y, xb[k][1].z, xb[k][1].w};
            const unsigned a2[4] = {xa[k][2].x, xa[k][2].y, xa[k][2].z, xa[k][2].w};
            const unsigned b2[4] = {xb[k][2].x, xb[k][2].y, xb[k][2].z, xb[k][2].w};
            int s0l = 0, s0h = 0, s1l = 0, s1h = 0, s2l = 0, s2h = 0;
#pragma unroll
            for (int t = 0; t < 4; t++) {
                unsigned lo = w[t] & 0x0f0f0f0fu;
                unsigned hi = (w[t] >> 4) & 0x0f0f0f0fu;
                if constexpr (FIVE) {  // qh byte i: bit 2c -> element i of sub-block 2c, 2c+1 -> 2c+1
                    const unsigned qh = t == 0 ? q5[j][k].x : t == 1 ? q5[j][k].y
                                      : t == 2 ? q5[j][k].z : q5[j][k].w;
                    lo |= ((qh >> (2 * c)) & 0x01010101u) << 4;
                    hi |= ((qh >> (2 * c + 1)) & 0x01010101u) << 4;
                } else if constexpr (SIX) {  // bits 2s, 2s+1 (low run) and 2s+4, 2s+5 (high run)
                    const unsigned qh = t == 0 ? q5[j][k].x : t == 1 ? q5[j][k].y
                                      : t == 2 ? q5[j][k].z : q5[j][k].w;
                    const unsigned q2 = qh >> sh6;
                    lo |= (q2 & 0x03030303u) << 4;
                    hi |= q2 & 0x30303030u;
                }
                s0l = dp4a_uu(lo, a0[t], s0l);
                s0h = dp4a_uu(hi, b0[t], s0h);
                s1l = dp4a_uu(lo, a1[t], s1l);
                s1h = dp4a_uu(hi, b1[t], s1h);
                s2l = dp4a_us(lo, a2[t], s2l);
                s2h = dp4a_us(hi, b2[t], s2h);
            }
            const float tl = fmaf((float)s2l, 65536.0f, (float)(s0l + 256 * s1l));
            const float th = fmaf((float)s2h, 65536.0f, (float)(s0h + 256 * s1h));
            if constexpr (SIX) {
                const float slo = (float)(int)(signed char)(h4[j][k].x >> by6);
                const float shi = (float)(int)(signed char)(h4[j][k].y >> by6);
                const float v = fmaf(slo, fmaf(sbr[k], tl, -32.0f * xsl[k]),
                                     shi * fmaf(sbr[k], th, -32.0f * xsh[k]));
                acc[j] = fmaf(d6[j][k], v, acc[j]);
            } else {
                float alo, ahi, blo, bhi;
                kq_scales(h4[j][k], c, alo, ahi, blo, bhi);
                float v = fmaf(sbr[k], fmaf(alo, tl, ahi * th), acc[j]);
                v = fmaf(-blo, xsl[k], v);
                acc[j] = fmaf(-bhi, xsh[k], v);
            }
        }
    }
}

template <int LAYOUT, int PRO, int EPI, class CF>
__global__ void __launch_bounds__(256) k_sgemv(GemvArgs a, int S) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float red8[32];
    constexpr int WPR = CF::WPR, BPL = CF::BPL, RPW = CF::RPW, RC = CF::RC;
    constexpr int SW = gemv_sw<LAYOUT>(), PBB = gemv_pbb<LAYOUT>();
    constexpr bool KQ = layout_kq<LAYOUT>();
    const int nb = a.K / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long nchunks = ((long)a.N + RC - 1) / RC;
    const int mycount =
        blockIdx.x < nchunks ? (int)((nchunks - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    const GemvSmem L(RC, WPR, nb, PBB, gemv_sc_bytes<LAYOUT>(RC, nb), S, a.K, PRO == PRO_NORM);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    unsigned char* stages = smem + 128;
    const Q24 q = q24_carve(stages + (size_t)S * L.stage, nb);
    float* hbuf = reinterpret_cast<float*>(stages + (size_t)S * L.stage + L.q24);
    float* red = reinterpret_cast<float*>(stages + (size_t)S * L.stage + L.q24 + L.hbuf);

    auto issue = [&](int i) {  // chunk i of this CTA into stage i % S (thread 0 only)
        const long c = blockIdx.x + (long)i * gridDim.x;
        const int s = i % S;
        const long row0 = c * RC;
        const int rows = (int)min((long)RC, (long)a.N - row0);
        const unsigned pb = (unsigned)rows * nb * PBB, sb = (unsigned)gemv_sc_bytes<LAYOUT>(rows, nb);
        const uint64_t pol = l2_evict_first();
        fence_proxy_async();
        mbar_expect_tx(&bars[s], pb + sb);
        bulk_g2s_hint(stages + (size_t)s * L.stage, a.payload + (size_t)row0 * nb * PBB, pb,
                      &bars[s], pol);
        if constexpr (SW > 0 || LAYOUT == LAYOUT_Q6K)
            bulk_g2s_hint(stages + (size_t)s * L.stage + L.pay,
                          reinterpret_cast<const char*>(a.scales) + gemv_sc_off<LAYOUT>(row0, nb),
                          sb, &bars[s], pol);
    };
    if (tid == 0) {
        for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    // weight streaming starts before the dependency on the previous kernel
    if (tid == 0)
        for (int i = 0; i < S && i < mycount; i++) issue(i);
    pdl_trigger();
    pdl_wait();

    gemv_prologue<LAYOUT, PRO>(a, q, hbuf, red8);
    __syncthreads();
    // this lane's activation planes, kept in registers
    uint4 xa[BPL][3], xb[BPL][3];
    int cbr[BPL];
    float sbr[BPL];
    const int wsub = warp % WPR, slot = warp / WPR;
#pragma unroll
    for (int k = 0; k < BPL; k++) {
        const int b = wsub * 32 + lane + k * 32 * WPR;
        const bool in = b < nb;
#pragma unroll
        for (int p = 0; p < 3; p++) {
            xa[k][p] = in ? q.pl[(p * 2 + 0) * nb + b] : make_uint4(0, 0, 0, 0);
            xb[k][p] = in ? q.pl[(p * 2 + 1) * nb + b] : make_uint4(0, 0, 0, 0);
        }
        cbr[k] = in ? q.cb[b] : 0;
        sbr[k] = in ? q.sb[b] : 0.f;
    }
    // k-quants: sb * (sum of the unit's low-run / high-run integers), for the
    // sub-blocks' min terms; each unit sits at the same place in its
    // super-block for all of this lane's units (b % 8 == lane % 8), so the
    // scale/min pair it reads is fixed per lane: sub-blocks 2c and 2c+1
    float xsl[BPL], xsh[BPL];
    const int kc = (lane & 7) >> 1;
    if constexpr (KQ) {
#pragma unroll
        for (int k = 0; k < BPL; k++) {
            int sl = 0, sh = 0, tl = 0, th = 0, ul = 0, uh = 0;
            const unsigned a0[4] = {xa[k][0].x, xa[k][0].y, xa[k][0].z, xa[k][0].w};
            const unsigned b0[4] = {xb[k][0].x, xb[k][0].y, xb[k][0].z, xb[k][0].w};
            const unsigned a1[4] = {xa[k][1].x, xa[k][1].y, xa[k][1].z, xa[k][1].w};
            const unsigned b1[4] = {xb[k][1].x, xb[k][1].y, xb[k][1].z, xb[k][1].w};
            const unsigned a2[4] = {xa[k][2].x, xa[k][2].y, xa[k][2].z, xa[k][2].w};
            const unsigned b2[4] = {xb[k][2].x, xb[k][2].y, xb[k][2].z, xb[k][2].w};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                sl = dp4a_uu(0x01010101u, a0[t], sl);
                sh = dp4a_uu(0x01010101u, b0[t], sh);
                tl = dp4a_uu(0x01010101u, a1[t], tl);
                th = dp4a_uu(0x01010101u, b1[t], th);
                ul = dp4a_us(0x01010101u, a2[t], ul);
                uh = dp4a_us(0x01010101u, b2[t], uh);
            }
            xsl[k] = sbr[k] * (float)(sl + 256 * tl + 65536 * ul);
            xsh[k] = sbr[k] * (float)(sh + 256 * th + 65536 * uh);
        }
    }

    unsigned long long best = argmax_key_init();
    int failed = 0;
    for (int i = 0; i < mycount; i++) {
        const int s = i % S;
        const unsigned par = (unsigned)((i / S) & 1);
        const bool ok = mbar_wait(&bars[s], par, GEMV_WAIT_NS);
        if (__syncthreads_or(!ok)) {
            failed = i + 1;
            break;
        }
        const unsigned char* pay = stages + (size_t)s * L.stage;
        const unsigned char* scs = pay + L.pay;
        const long row0 = (blockIdx.x + (long)i * gridDim.x) * RC;
        const int rows = (int)min((long)RC, (long)a.N - row0);
        float* rb = red + (size_t)(i & 1) * RC * WPR;
        float acc[RPW];
        if constexpr (LAYOUT == LAYOUT_Q8) {
            // int8 codes (32 bytes per block: elements 0-15 pair with the
            // low planes, 16-31 with the high ones) times the q24 planes:
            // sum q X = D0 + 256 D1 + 65536 D2, q signed
            uint4 wa[RPW][BPL], wb[RPW][BPL];
            float dd[RPW][BPL];
#pragma unroll
            for (int j = 0; j < RPW; j++) {
                const int r = slot * RPW + j;
#pragma unroll
                for (int k = 0; k < BPL; k++) {
                    const int b = wsub * 32 + lane + k * 32 * WPR;
                    const bool in = r < rows && b < nb;
                    const size_t blk = in ? (size_t)r * nb + b : 0;
                    const uint4 z = make_uint4(0, 0, 0, 0);
                    wa[j][k] = in ? reinterpret_cast<const uint4*>(pay)[2 * blk] : z;
                    wb[j][k] = in ? reinterpret_cast<const uint4*>(pay)[2 * blk + 1] : z;
                    dd[j][k] = in ? __half2float(reinterpret_cast<const __half*>(scs)[blk]) : 0.f;
                }
            }
#pragma unroll
            for (int j = 0; j < RPW; j++) {
                acc[j] = 0.f;
#pragma unroll
                for (int k = 0; k < BPL; k++) {
                    const unsigned lo[4] = {wa[j][k].x, wa[j][k].y, wa[j][k].z, wa[j][k].w};
                    const unsigned hi[4] = {wb[j][k].x, wb[j][k].y, wb[j][k].z, wb[j][k].w};
                    const unsigned a0[4] = {xa[k][0].x, xa[k][0].y, xa[k][0].z, xa[k][0].w};
                    const unsigned b0[4] = {xb[k][0].x, xb[k][0].y, xb[k][0].z, xb[k][0].w};
                    const unsigned a1[4] = {xa[k][1].x, xa[k][1].y, xa[k][1].z, xa[k][1].w};
                    const unsigned b1[4] = {xb[k][1].x, xb[k][1].y, xb[k][1].z, xb[k][1].w};
                    const unsigned a2[4] = {xa[k][2].x, xa[k][2].y, xa[k][2].z, xa[k][2].w};
                    const unsigned b2[4] = {xb[k][2].x, xb[k][2].y, xb[k][2].z, xb[k][2].w};
                    int s0l = 0, s0h = 0, s1l = 0, s1h = 0, s2l = 0, s2h = 0;
#pragma unroll
                    for (int t = 0; t < 4; t++) {
                        s0l = dp4a_su(lo[t], a0[t], s0l);
                        s0h = dp4a_su(hi[t], b0[t], s0h);
                        s1l = dp4a_su(lo[t], a1[t], s1l);
                        s1h = dp4a_su(hi[t], b1[t], s1h);
                        s2l = dp4a_ss(lo[t], a2[t], s2l);
                        s2h = dp4a_ss(hi[t], b2[t], s2h);
                    }
                    const int s01 = (s0l + s0h) + (s1l + s1h) * 256;
                    const float T = fmaf((float)(s2l + s2h), 65536.0f, (float)s01);
                    acc[j] = fmaf(dd[j][k] * sbr[k], T, acc[j]);
                }
            }
        } else if constexpr (KQ) {
            kq_chunk<LAYOUT, RPW, BPL, WPR>(pay, scs, nb, rows, slot, wsub, lane, kc, xa, xb, sbr,
                                            xsl, xsh, acc);
        } else {
        // all of this warp's loads first (RPW rows x BPL blocks), then the math
        uint4 w4[RPW][BPL];
        float dd[RPW][BPL];
#pragma unroll
        for (int j = 0; j < RPW; j++) {
            const int r = slot * RPW + j;
#pragma unroll
            for (int k = 0; k < BPL; k++) {
                const int b = wsub * 32 + lane + k * 32 * WPR;
                const bool in = r < rows && b < nb;
                const size_t blk = in ? (size_t)r * nb + b : 0;
                w4[j][k] = in ? reinterpret_cast<const uint4*>(pay)[blk] : make_uint4(0, 0, 0, 0);
                dd[j][k] = !in ? 0.f
                               : (SW == 2 ? __half2float(reinterpret_cast<const __half*>(scs)[blk])
                                          : reinterpret_cast<const float*>(scs)[blk]);
            }
        }
#pragma unroll
        for (int j = 0; j < RPW; j++) {
            acc[j] = 0.f;
#pragma unroll
            for (int k = 0; k < BPL; k++) {
                const unsigned w[4] = {w4[j][k].x, w4[j][k].y, w4[j][k].z, w4[j][k].w};
                const unsigned a0[4] = {xa[k][0].x, xa[k][0].y, xa[k][0].z, xa[k][0].w};
                const unsigned b0[4] = {xb[k][0].x, xb[k][0].y, xb[k][0].z, xb[k][0].w};
                const unsigned a1[4] = {xa[k][1].x, xa[k][1].y, xa[k][1].z, xa[k][1].w};
                const unsigned b1[4] = {xb[k][1].x, xb[k][1].y, xb[k][1].z, xb[k][1].w};
                const unsigned a2[4] = {xa[k][2].x, xa[k][2].y, xa[k][2].z, xa[k][2].w};
                const unsigned b2[4] = {xb[k][2].x, xb[k][2].y, xb[k][2].z, xb[k][2].w};
                // six independent dp4a chains of four (low / high nibbles apart)
                int s0l = 0, s0h = 0, s1l = 0, s1h = 0, s2l = 0, s2h = 0;
#pragma unroll
                for (int t = 0; t < 4; t++) {
                    const unsigned lo = w[t] & 0x0f0f0f0fu;
                    const unsigned hi = (w[t] >> 4) & 0x0f0f0f0fu;
                    s0l = dp4a_uu(lo, a0[t], s0l);
                    s0h = dp4a_uu(hi, b0[t], s0h);
                    s1l = dp4a_uu(lo, a1[t], s1l);
                    s1h = dp4a_uu(hi, b1[t], s1h);
                    s2l = dp4a_us(lo, a2[t], s2l);
                    s2h = dp4a_us(hi, b2[t], s2h);
                }
                const int s01 = (s0l + s0h) + ((s1l + s1h) << 8) - cbr[k];
                const float T = fmaf((float)(s2l + s2h), 65536.0f, (float)s01);
                acc[j] = fmaf(dd[j][k] * sbr[k], T, acc[j]);
            }
        }
        }
        // transposed butterfly: the RPW row sums in 5 shuffles; afterwards lane
        // (32/RPW)*j holds the warp's partial of row slot*RPW + j
        float v = warp_reduce_rows<RPW>(acc, lane);
        if ((lane & (32 / RPW - 1)) == 0) rb[(slot * RPW + lane / (32 / RPW)) * WPR + wsub] = v;
        __syncthreads();  // stage s consumed, row partials complete
        if (tid == 0 && i + S < mycount) issue(i + S);
        // epilogue: fixed-order sum of the WPR partials of each row
        if (EPI == EPI_GLU) {
            if (tid < RC / 2) {
                const int r0 = 2 * tid;
                if (r0 + 1 < rows) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int w = 0; w < WPR; w++) {
                        gv += rb[r0 * WPR + w];
                        uv += rb[(r0 + 1) * WPR + w];
                    }
                    const float act = a.geglu ? gelu_ref_f(gv) : silu_ref_f(gv);
                    a.y[(row0 + r0) / 2] = act * uv;
                }
            }
        } else if (tid < RC && tid < rows) {
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < WPR; w++) v += rb[tid * WPR + w];
            const long row = row0 + tid;
            if (EPI == EPI_RESID) {
                a.y[row] = a.y[row] + v;
            } else if (EPI == EPI_HEAD) {
                if (a.softcap > 0.f) v = a.softcap * tanhf(v / a.softcap);
                a.y[row] = v;
                const unsigned long long kk = argmax_key(v, (unsigned)row + a.key_offset);
                best = kk > best ? kk : best;
            } else {
                a.y[row] = a.bias ? v + a.bias[row] : v;
            }
        }
    }
    if (failed) {
        // record the timeout and let every issued copy land before exiting
        if (tid == 0) {
            atomicExch(a.status, (int)DEV_TIMEOUT);
            const int issued = min(mycount, failed - 1 + S);
            for (int i = failed - 1; i < issued; i++)
                mbar_wait(&bars[i % S], (unsigned)((i / S) & 1), GEMV_WAIT_NS);
        }
        return;
    }
    if (EPI == EPI_HEAD && warp == 0) {  // RC <= 32: the epilogue rows live in warp 0
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long t = __shfl_xor_sync(FULL, best, o);
            best = t > best ? t : best;
        }
        if (lane == 0 && mycount > 0) atomicMax(a.key, best);
    }
}

// ---- host side ----------------------------------------------------------------
// The streaming kernel handles K with K/32 a multiple of 8 (GGUF f16 scales,
// whole k-quant super-blocks) or 4 (crate f32 scales), so every chunk copy is
// a multiple of 16 bytes, and K <= 24576.
inline bool sgemv_supported(int layout, int K) {
    const int nb = K / 32;
    if (K % 32 || nb > GemvC768::NB_MAX) return false;
    if (layout == LAYOUT_REF) return nb % 4 == 0;
    if (nb % 8) return false;
    if (layout == LAYOUT_Q6K) {  // every chunk's d values start 16-byte aligned: RC * nb/8 % 8 == 0
        const int rc = nb <= GemvC96::NB_MAX ? 16 : nb <= GemvC192::NB_MAX ? 8
                     : nb <= GemvC384::NB_MAX ? 4 : 1;
        return (rc * (nb / 8)) % 8 == 0;
    }
    return true;
}

int launch_sgemv(cw_ctx* ctx, int layout, int pro, int epi, const GemvArgs& a, bool pdl);

}  // namespace cw
