// cw_device.cuh -- device building blocks shared by the op kernels and the
// fused decode kernels.
//
// Q4 dot products run on the integer dot-product unit.  The activation
// vector x is converted once per CTA into a block-floating-point form ("q24"):
// per 32-element block b, an exponent e_b with max|x| < 2^e_b and integers
// X_j = rn(x_j * 2^(22-e_b)), |X_j| <= 2^22, split into three byte planes
// X = X0 + 256*X1 + 65536*X2 (X0, X1 unsigned, X2 signed).  A weight block's
// 4-bit codes q_j (0..15) then give
//     sum_j (q_j - 8) * X_j = dp4a(q, X0) + 256*dp4a(q, X1) + 65536*dp4a(q, X2)
//                             - 8 * sum_j X_j
// exactly in integers, and the block contributes d_b * 2^(e_b-22) times that.
// The only rounding is x -> X (relative 2^-23 of the block maximum) and the
// final f32 combine, which keeps the GEMV within f32-accumulation accuracy of
// the reference's sum_k x_k * (d*(q_k-8)) (src/kernels/q4.wgsl:25-82,
// src/kernels/matmul.wgsl:43-50) while spending ~1.4 instructions per weight
// instead of ~3 for a float unpack + FFMA.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace cw {

constexpr unsigned FULL = 0xffffffffu;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

// d = c + sum_i a.u8[i] * b.u8[i]
__device__ __forceinline__ int dp4a_uu(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// d = c + sum_i a.u8[i] * b.s8[i]
__device__ __forceinline__ int dp4a_us(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// d = c + sum_i a.s8[i] * b.u8[i]
__device__ __forceinline__ int dp4a_su(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// d = c + sum_i a.s8[i] * b.s8[i]
__device__ __forceinline__ int dp4a_ss(unsigned a, unsigned b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Streaming 16-byte load of read-once weight data: bypass L1.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ unsigned short ldg_u16(const void* p) {
    unsigned short r;
    asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}

// ---- programmatic dependent launch (PDL) -----------------------------------
// A kernel launched with programmatic stream serialisation may start before
// its predecessor finishes; pdl_wait() blocks until the predecessor grid has
// completed and its writes are visible, pdl_trigger() lets the successor
// start launching.  Both are no-ops for a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Hint the bytes [lo, hi) of a read-only buffer into L2 with bulk prefetches
// issued by the calling thread.  lo is rounded down and hi up to 16 bytes;
// callers pass ranges inside allocations that are 256-byte aligned and
// padded, so the rounded range stays inside the allocation.
__device__ __forceinline__ void prefetch_l2(const void* lo, const void* hi) {
    uintptr_t a = reinterpret_cast<uintptr_t>(lo) & ~uintptr_t(15);
    uintptr_t b = (reinterpret_cast<uintptr_t>(hi) + 15) & ~uintptr_t(15);
    while (a < b) {
        uint32_t n = (b - a) > (1u << 20) ? (1u << 20) : (uint32_t)(b - a);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a), "r"(n) : "memory");
        a += n;
    }
}

// Weight layouts understood by the GEMV core.
enum Q4Layout : int {
    // GGUF Q4_0 repacked into planes: nibble payload [rows][nb][16] (byte j:
    // low nibble = element j, high nibble = element j+16, dequant.rs:70-75)
    // and f16 scales [rows][nb].
    LAYOUT_GGUF = 0,
    // chat-wgpu's re-quantised layout (q4.rs:32-36): u32 quants, nibble n of
    // word w of block b = element b*32 + w*8 + n; f32 scales [rows][nb].
    LAYOUT_REF = 1,
    // Raw GGUF Q4_K / Q5_K super-blocks [rows][K/256][144 | 176] (d, dmin,
    // 12 bytes of 6-bit scales/mins, Q5_K's 32 fifth-bit bytes, 128 nibble
    // bytes).  The GEMV takes each 16-byte run of nibbles as one "unit":
    // run u of a super-block (chunk c = u/2, half h = u%2) holds elements
    // 64c + 16h + i (low nibbles, sub-block 2c) and 64c + 32 + 16h + i (high
    // nibbles, sub-block 2c+1), i < 16.
    LAYOUT_Q4K = 2,
    LAYOUT_Q5K = 3,
    // GGUF Q6_K split into 16-byte-aligned planes (the file's 210-byte
    // super-blocks are 2-byte aligned): [rows][K/256][208] = ql[128] qh[64]
    // scales[16] as in the file, then the f16 d of every super-block
    // [rows][K/256].  Unit u of a super-block (half h = u/4, s = (u/2)%2,
    // t = u%2) is ql bytes 16u..16u+15: low nibbles elements 128h + 32s +
    // 16t + i (scale 8h + 2s + t), high nibbles the same + 64 (scale + 4);
    // their top two bits are bits 2s and 2s+4 of qh[32h + 16t + i].
    LAYOUT_Q6K = 4,
    // GGUF Q8_0 split like Q4_0: int8 codes [rows][nb][32] (byte j = element
    // j of the block) and f16 scales [rows][nb].
    LAYOUT_Q8 = 5,
};

template <int LAYOUT>
__host__ __device__ constexpr bool layout_kq() {
    return LAYOUT == LAYOUT_Q4K || LAYOUT == LAYOUT_Q5K || LAYOUT == LAYOUT_Q6K;
}

// Element of x that element e (0..31) of GEMV unit b pairs with: the unit's
// 32-element block for Q4_0 planes; for the k-quant layouts, the unit's low
// run (e < 16) and high run (e >= 16), 32 elements apart (Q6_K: 64).
template <int LAYOUT>
__device__ __forceinline__ int unit_elem(int b, int e) {
    if constexpr (LAYOUT == LAYOUT_Q6K) {
        const int u = b & 7;
        return (b >> 3) * 256 + 128 * (u >> 2) + 32 * ((u >> 1) & 1) + 16 * (u & 1) + (e & 15) +
               ((e & 16) << 2);
    } else if constexpr (layout_kq<LAYOUT>()) {
        return (b >> 1) * 64 + 16 * (b & 1) + (e & 15) + ((e & 16) << 1);
    } else {
        return b * 32 + e;
    }
}

// Byte position, inside a block's 32-byte plane row, of block element j.
// Words 0-3 pair with the low nibbles of payload words 0-3, words 4-7 with
// their high nibbles (after `>> 4`).
template <int LAYOUT>
__device__ __forceinline__ int q24_pos(int j) {
    if (LAYOUT == LAYOUT_GGUF) return j;
    int w = j >> 3, i = (j & 7) >> 1, par = j & 1;
    return (par ? 16 : 0) + 4 * w + i;
}

// q24 activation planes in shared memory for nb blocks.
//   pl : uint4 [3 planes][2 halves][nb]  (plane row of block b: halves 0,1)
//   cb : int   [nb]   8 * sum_j X_j
//   sb : float [nb]   2^(e_b-22); 0 for an all-zero block; NaN if the block
//                      holds a non-finite value (the output becomes NaN)
struct Q24 {
    uint4* pl;
    int* cb;
    float* sb;
    int nb;
};

__host__ __device__ constexpr size_t q24_bytes(int nb) { return (size_t)nb * (96 + 8); }

__device__ __forceinline__ Q24 q24_carve(void* smem, int nb) {
    Q24 q;
    q.pl = reinterpret_cast<uint4*>(smem);
    q.cb = reinterpret_cast<int*>(reinterpret_cast<char*>(smem) + (size_t)nb * 96);
    q.sb = reinterpret_cast<float*>(reinterpret_cast<char*>(smem) + (size_t)nb * 100);
    q.nb = nb;
    return q;
}

// Block exponent and this lane's 24-bit integer from the block's max |v|
// given as IEEE bits (mbits >= 0x7f800000: the block holds Inf/NaN).  For a
// normal max with exponent field e >= 22, frexp's E is e - 126 and both
// 2^(22-E) and 2^(E-22) are normal floats built from their exponent fields,
// so v * 2^(22-E) is exact and equals ldexpf(v, 22 - E); smaller maxima take
// the frexpf/ldexpf path.
__device__ __forceinline__ void q24_scale(unsigned mbits, float v, int& X, float& sb) {
    X = 0;
    if (mbits >= 0x7f800000u) {
        sb = __int_as_float(0x7fc00000);
    } else if (mbits == 0u) {
        sb = 0.0f;
    } else {
        const unsigned e = mbits >> 23;
        if (e >= 22u) {
            X = __float2int_rn(v * __uint_as_float((275u - e) << 23));
            sb = __uint_as_float((e - 21u) << 23);
        } else {
            int E;
            frexpf(__uint_as_float(mbits), &E);  // m = f * 2^E, f in [0.5, 1)
            X = __float2int_rn(ldexpf(v, 22 - E));
            sb = ldexpf(1.0f, E - 22);
        }
    }
}

// Convert one 32-element block held one element per lane (v) into the planes.
// The block max and the sum of the integers are single-instruction warp
// reductions (redux.sync): for non-negative floats the IEEE bit patterns
// order like the values, and Inf/NaN compare above every finite value.
template <int LAYOUT>
__device__ __forceinline__ void q24_block(const Q24& s, int b, float v, int lane) {
    const unsigned mbits = __reduce_max_sync(FULL, __float_as_uint(fabsf(v)));
    int X;
    float sb;
    q24_scale(mbits, v, X, sb);
    int pos = q24_pos<LAYOUT>(lane);
    uint8_t* base = reinterpret_cast<uint8_t*>(s.pl);
    int half = pos >> 4, off = pos & 15;
#pragma unroll
    for (int p = 0; p < 3; p++) {
        int byte = (p == 2) ? ((X >> 16) & 0xff) : ((X >> (8 * p)) & 0xff);
        base[((size_t)(p * 2 + half) * s.nb + b) * 16 + off] = (uint8_t)byte;
    }
    const int sx = __reduce_add_sync(FULL, X);
    if (lane == 0) {
        s.cb[b] = 8 * sx;
        s.sb[b] = sb;
    }
}

// The same planes from four consecutive elements per lane (GGUF layout only):
// lane L of a warp covers block b = (quad group) * 4 + L/8, elements
// 4*(L%8) .. 4*(L%8)+3, given as one float4.  The block max and the integer
// sum are 3-step shuffles within the 8 lanes of a block, and each lane
// writes one 32-bit word per byte plane (its 4 elements' bytes, packed with
// __byte_perm): the bytes q24_block<LAYOUT_GGUF> writes, in a quarter of
// the instructions.  `valid` (b < nb) may differ between the warp's four
// groups; every lane takes part in the shuffles.
__device__ __forceinline__ void q24_quad(const Q24& s, int b, bool valid, const float4& v,
                                         int lane) {
    unsigned m = max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
                     max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w))));
    m = max(m, __shfl_xor_sync(FULL, m, 1));
    m = max(m, __shfl_xor_sync(FULL, m, 2));
    m = max(m, __shfl_xor_sync(FULL, m, 4));
    int X0, X1, X2, X3;
    float sb;
    q24_scale(m, v.x, X0, sb);
    q24_scale(m, v.y, X1, sb);
    q24_scale(m, v.z, X2, sb);
    q24_scale(m, v.w, X3, sb);
    const int g8 = lane & 7, half = g8 >> 2, w = g8 & 3;
    if (valid) {
        uint32_t* pw = reinterpret_cast<uint32_t*>(s.pl);
#pragma unroll
        for (int pl = 0; pl < 3; pl++) {
            const unsigned sel = (unsigned)pl | ((4u + pl) << 4);
            const unsigned lo = __byte_perm((unsigned)X0, (unsigned)X1, sel);
            const unsigned hi = __byte_perm((unsigned)X2, (unsigned)X3, sel);
            pw[((size_t)(pl * 2 + half) * s.nb + b) * 4 + w] = __byte_perm(lo, hi, 0x5410);
        }
    }
    int sx = (X0 + X1) + (X2 + X3);
    sx += __shfl_xor_sync(FULL, sx, 1);
    sx += __shfl_xor_sync(FULL, sx, 2);
    sx += __shfl_xor_sync(FULL, sx, 4);
    if (valid && g8 == 0) {
        s.cb[b] = 8 * sx;
        s.sb[b] = sb;
    }
}

// Whole vector from global/shared f32 x[K]; all threads of the CTA call it,
// a __syncthreads() must follow before the planes are read.
template <int LAYOUT>
__device__ void q24_prepare(const Q24& s, const float* x) {
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    for (int b = warp; b < s.nb; b += nw) q24_block<LAYOUT>(s, b, x[b * 32 + lane], lane);
}

// Accumulate R consecutive weight rows [row0, row0+R) against the q24 vector:
// lane l takes blocks l, l+32, ...  acc[r] gets this lane's partial; the
// caller reduces across the warp.  Rows >= nrows are skipped (acc untouched).
//   payload : LAYOUT_GGUF -> uint8 [rows][nb][16];  LAYOUT_REF -> u32 [rows][nb*4]
//   scales  : LAYOUT_GGUF -> __half [rows][nb];      LAYOUT_REF -> float [rows][nb]
template <int LAYOUT, int R>
__device__ __forceinline__ void q4_rows_dot(const Q24& s, const uint8_t* __restrict__ payload,
                                            const void* __restrict__ scales, long row0, long nrows,
                                            int lane, float (&acc)[R]) {
    const int nb = s.nb;
    for (int b = lane; b < nb; b += 32) {
        uint4 q[R];
        float d[R];
#pragma unroll
        for (int r = 0; r < R; r++) {
            long row = row0 + r;
            if (row >= nrows) row = nrows - 1;  // clamp: loaded but never used
            size_t blk = (size_t)row * nb + b;
            q[r] = ldg_stream(payload + blk * 16);
            if (LAYOUT == LAYOUT_GGUF)
                d[r] = __half2float(__ushort_as_half(
                    ldg_u16(reinterpret_cast<const unsigned short*>(scales) + blk)));
            else
                d[r] = __ldg(reinterpret_cast<const float*>(scales) + blk);
        }
        const uint4 x0a = s.pl[(0 * 2 + 0) * nb + b], x0b = s.pl[(0 * 2 + 1) * nb + b];
        const uint4 x1a = s.pl[(1 * 2 + 0) * nb + b], x1b = s.pl[(1 * 2 + 1) * nb + b];
        const uint4 x2a = s.pl[(2 * 2 + 0) * nb + b], x2b = s.pl[(2 * 2 + 1) * nb + b];
        const int cb = s.cb[b];
        const float sb = s.sb[b];
#pragma unroll
        for (int r = 0; r < R; r++) {
            int s0 = 0, s1 = 0, s2 = 0;
            const unsigned w[4] = {q[r].x, q[r].y, q[r].z, q[r].w};
            const unsigned a0[4] = {x0a.x, x0a.y, x0a.z, x0a.w}, b0[4] = {x0b.x, x0b.y, x0b.z, x0b.w};
            const unsigned a1[4] = {x1a.x, x1a.y, x1a.z, x1a.w}, b1[4] = {x1b.x, x1b.y, x1b.z, x1b.w};
            const unsigned a2[4] = {x2a.x, x2a.y, x2a.z, x2a.w}, b2[4] = {x2b.x, x2b.y, x2b.z, x2b.w};
#pragma unroll
            for (int t = 0; t < 4; t++) {
                unsigned lo = w[t] & 0x0f0f0f0fu;
                unsigned hi = (w[t] >> 4) & 0x0f0f0f0fu;
                s0 = dp4a_uu(lo, a0[t], s0);
                s0 = dp4a_uu(hi, b0[t], s0);
                s1 = dp4a_uu(lo, a1[t], s1);
                s1 = dp4a_uu(hi, b1[t], s1);
                s2 = dp4a_us(lo, a2[t], s2);
                s2 = dp4a_us(hi, b2[t], s2);
            }
            float T = fmaf((float)s2, 65536.0f, (float)(s0 + (s1 << 8) - cb));
            acc[r] = fmaf(d[r] * sb, T, acc[r]);
        }
    }
}

// f32 <-> order-preserving u32 key (for a packed argmax via atomicMax).
__device__ __forceinline__ unsigned f32_order_key(float f) {
    unsigned u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Argmax key: larger = better; ties resolve to the lowest index because the
// index is stored inverted (argmax.wgsl:26,43 tie rule).  NaN never wins.
__device__ __forceinline__ unsigned long long argmax_key(float v, unsigned idx) {
    if (v != v) return 0ull;
    if (v == 0.0f) v = 0.0f;  // -0 and +0 compare equal in the reference's '>' scan
    return ((unsigned long long)f32_order_key(v) << 32) | (unsigned long long)(~idx);
}
// The reference's start value: best = -3.402823e38 with index 0, so nothing
// at or below it wins and the answer is then 0 (argmax.wgsl:23,30-31).
__device__ __forceinline__ unsigned long long argmax_key_init() {
    return argmax_key(-3.402823e38f, 0u);
}
__device__ __forceinline__ unsigned argmax_key_index(unsigned long long k) {
    return ~(unsigned)(k & 0xffffffffull);
}

}  // namespace cw
