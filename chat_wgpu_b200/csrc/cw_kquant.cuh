// cw_kquant.cuh -- device code of the GGUF weight formats kept raw in HBM:
// the k-quants (Q4_K, Q5_K, Q6_K super-blocks of 256 weights) and the other
// types the reference's loader takes (F32, F16, Q4_1, Q8_0: tensor_f32,
// src/loader/gguf.rs:109-121) plus BF16, each read 256 weights at a time
// (a "group": one super-block, or 8 blocks of 32).  Per-lane dequantisation
// and dot products shared by the raw-weight GEMV (cw_kquant.cu) and the
// model's projections, embedding rows and LM heads (cw_model.cu).
//
// Q6_K follows the reference's dequant_q6_k (src/loader/dequant.rs:102-131):
// w = (d * sc) * (q - 32), f32, left to right; Q8_0 dequant_q8_0 (:46-58)
// w = d * q; Q4_1 dequant_q4_1 (:82-97) w = d * q + m; F16 f16_to_f32
// (:9-21).  Q4_K / Q5_K are not in the reference (dequant.rs:6,
// ROADMAP.md:52-53); they restate ggml's published block_q4_K / block_q5_K
// layout: w = (d * sc) * q - (dmin * m).  BF16 is the top half of an f32
// (dequant_bf16, dequant.rs:41-43, which the reference's tensor_f32 does not
// dispatch).  Each formula is evaluated in the stated order with
// one f32 rounding per operation (no contraction), so dequantised values are
// exact to it.  The GEMV dot products group the same terms differently
// (d * sum(q x) instead of sum((d q) x)): f32-accumulation grade.
#pragma once

#include <stdint.h>

#include "cw_common.h"
#include "cw_device.cuh"

namespace cw {


// Bytes of one 256-weight group and raw words one lane loads per group.
template <int T>
struct KQ;
template <>
struct KQ<CW_GGUF_Q4_K> {
    static constexpr int BYTES = 144, WORDS = 6;
};
template <>
struct KQ<CW_GGUF_Q5_K> {
    static constexpr int BYTES = 176, WORDS = 6;
};
template <>
struct KQ<CW_GGUF_Q6_K> {
    static constexpr int BYTES = 210, WORDS = 6;
};
template <>
struct KQ<CW_GGUF_F32> {
    static constexpr int BYTES = 1024, WORDS = 8;
};
template <>
struct KQ<CW_GGUF_F16> {
    static constexpr int BYTES = 512, WORDS = 4;
};
template <>
struct KQ<CW_GGUF_BF16> {
    static constexpr int BYTES = 512, WORDS = 4;
};
template <>
struct KQ<CW_GGUF_Q8_0> {  // 8 blocks of 34 bytes: f16 d, 32 x int8
    static constexpr int BYTES = 272, WORDS = 3;
};
template <>
struct KQ<CW_GGUF_Q4_1> {  // 8 blocks of 20 bytes: f16 d, f16 m, 16 nibble bytes
    static constexpr int BYTES = 160, WORDS = 2;
};
// The formats whose 8 weights per lane are 8 consecutive elements (lane l:
// elements 8l .. 8l+7 of the group): the plain float types and Q8_0.
template <int T>
constexpr bool kq_consecutive() {
    return T == CW_GGUF_F32 || T == CW_GGUF_F16 || T == CW_GGUF_BF16 || T == CW_GGUF_Q8_0;
}

__device__ __forceinline__ float kq_bf16(uint32_t bits16) {
    return __uint_as_float((bits16 & 0xffffu) << 16);
}

__device__ __forceinline__ float kq_f16(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

__device__ __forceinline__ void kq_scale_min(int j, const uint8_t* q, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// The 8 weights lane `lane` owns in super-block `blk`: values w[8] and their
// indices within the block idx[8].
template <int T>
__device__ __forceinline__ void kq_lane(const uint8_t* __restrict__ blk, int lane, float (&w)[8],
                                        int (&idx)[8]) {
    if constexpr (T == CW_GGUF_F32) {
#pragma unroll
        for (int i = 0; i < 8; i++) {
            w[i] = reinterpret_cast<const float*>(blk)[8 * lane + i];
            idx[i] = 8 * lane + i;
        }
    } else if constexpr (T == CW_GGUF_F16 || T == CW_GGUF_BF16) {
        const uint16_t* h = reinterpret_cast<const uint16_t*>(blk) + 8 * lane;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            w[i] = T == CW_GGUF_F16 ? kq_f16(blk + 2 * (8 * lane + i)) : kq_bf16(h[i]);
            idx[i] = 8 * lane + i;
        }
    } else if constexpr (T == CW_GGUF_Q8_0) {
        const int c = lane >> 2, j0 = 8 * (lane & 3);
        const uint8_t* b = blk + 34 * c;
        const float d = kq_f16(b);
#pragma unroll
        for (int i = 0; i < 8; i++) {
            w[i] = __fmul_rn(d, (float)(int8_t)b[2 + j0 + i]);
            idx[i] = 32 * c + j0 + i;
        }
    } else if constexpr (T == CW_GGUF_Q4_1) {
        const int c = lane >> 2, j0 = 4 * (lane & 3);
        const uint8_t* b = blk + 20 * c;
        const float d = kq_f16(b), m = kq_f16(b + 2);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int q = b[4 + j0 + i];
            w[i] = __fadd_rn(__fmul_rn(d, (float)(q & 0x0f)), m);
            w[4 + i] = __fadd_rn(__fmul_rn(d, (float)(q >> 4)), m);
            idx[i] = 32 * c + j0 + i;
            idx[4 + i] = 32 * c + 16 + j0 + i;
        }
    } else if constexpr (T == CW_GGUF_Q6_K) {
        const int h = lane >> 4, l0 = 2 * (lane & 15), is = l0 >> 4;
        const uint8_t* ql = blk + 64 * h;
        const uint8_t* qh = blk + 128 + 32 * h;
        const int8_t* sc = (const int8_t*)(blk + 192 + 8 * h);
        const float d = kq_f16(blk + 208);
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int l = l0 + u;
            const int a = ql[l], b = ql[l + 32], hb = qh[l];
            const int q1 = ((a & 0x0f) | (((hb >> 0) & 3) << 4)) - 32;
            const int q2 = ((b & 0x0f) | (((hb >> 2) & 3) << 4)) - 32;
            const int q3 = ((a >> 4) | (((hb >> 4) & 3) << 4)) - 32;
            const int q4 = ((b >> 4) | (((hb >> 6) & 3) << 4)) - 32;
            w[4 * u + 0] = __fmul_rn(__fmul_rn(d, (float)sc[is + 0]), (float)q1);
            w[4 * u + 1] = __fmul_rn(__fmul_rn(d, (float)sc[is + 2]), (float)q2);
            w[4 * u + 2] = __fmul_rn(__fmul_rn(d, (float)sc[is + 4]), (float)q3);
            w[4 * u + 3] = __fmul_rn(__fmul_rn(d, (float)sc[is + 6]), (float)q4);
            idx[4 * u + 0] = 128 * h + l;
            idx[4 * u + 1] = 128 * h + l + 32;
            idx[4 * u + 2] = 128 * h + l + 64;
            idx[4 * u + 3] = 128 * h + l + 96;
        }
    } else {
        constexpr bool five = T == CW_GGUF_Q5_K;
        const int c = lane >> 3, j0 = 4 * (lane & 7);
        const float d = kq_f16(blk), dmin = kq_f16(blk + 2);
        const uint8_t* scales = blk + 4;
        const uint8_t* qs = blk + (five ? 48 : 16) + 32 * c + j0;
        int sc1, m1, sc2, m2;
        kq_scale_min(2 * c, scales, &sc1, &m1);
        kq_scale_min(2 * c + 1, scales, &sc2, &m2);
        const float d1 = __fmul_rn(d, (float)sc1), mm1 = __fmul_rn(dmin, (float)m1);
        const float d2 = __fmul_rn(d, (float)sc2), mm2 = __fmul_rn(dmin, (float)m2);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            int lo = qs[i] & 0x0f, hi = qs[i] >> 4;
            if constexpr (five) {
                const int hb = blk[16 + j0 + i];
                lo += ((hb >> (2 * c)) & 1) << 4;
                hi += ((hb >> (2 * c + 1)) & 1) << 4;
            }
            w[i] = __fsub_rn(__fmul_rn(d1, (float)lo), mm1);
            w[4 + i] = __fsub_rn(__fmul_rn(d2, (float)hi), mm2);
            idx[i] = 64 * c + j0 + i;
            idx[4 + i] = 64 * c + 32 + j0 + i;
        }
    }
}

// Raw words one lane needs from a super-block, loaded ahead of the math so
// several blocks' loads are in flight at once.
template <int T>
struct KqRaw {
    uint32_t v[KQ<T>::WORDS];
};

template <int T>
__device__ __forceinline__ KqRaw<T> kq_load(const uint8_t* __restrict__ blk, int lane) {
    KqRaw<T> r;
    if constexpr (T == CW_GGUF_F32) {  // 32 bytes at 32*lane (group starts are 16-byte aligned)
        const uint4* b4 = reinterpret_cast<const uint4*>(blk) + 2 * lane;
        const uint4 a = __ldg(b4), b = __ldg(b4 + 1);
        r.v[0] = a.x; r.v[1] = a.y; r.v[2] = a.z; r.v[3] = a.w;
        r.v[4] = b.x; r.v[5] = b.y; r.v[6] = b.z; r.v[7] = b.w;
    } else if constexpr (T == CW_GGUF_F16 || T == CW_GGUF_BF16) {  // 16 bytes at 16*lane
        const uint4 a = __ldg(reinterpret_cast<const uint4*>(blk) + lane);
        r.v[0] = a.x; r.v[1] = a.y; r.v[2] = a.z; r.v[3] = a.w;
    } else if constexpr (T == CW_GGUF_Q8_0) {  // block lane/4 (2-byte aligned): d, 8 codes
        const uint16_t* b16 = reinterpret_cast<const uint16_t*>(blk + 34 * (lane >> 2));
        const int o = 1 + 4 * (lane & 3);  // u16 index of the lane's first code pair
        r.v[0] = __ldg(b16 + o) | ((uint32_t)__ldg(b16 + o + 1) << 16);
        r.v[1] = __ldg(b16 + o + 2) | ((uint32_t)__ldg(b16 + o + 3) << 16);
        r.v[2] = __ldg(b16);
    } else if constexpr (T == CW_GGUF_Q4_1) {  // block lane/4 (4-byte aligned): d|m, 4 bytes
        const uint32_t* b32 = reinterpret_cast<const uint32_t*>(blk + 20 * (lane >> 2));
        r.v[0] = __ldg(b32);
        r.v[1] = __ldg(b32 + 1 + (lane & 3));
    } else if constexpr (T == CW_GGUF_Q6_K) {  // 210-byte blocks: 2-byte alignment
        const int h = lane >> 4, l0 = 2 * (lane & 15);
        const uint16_t* b16 = (const uint16_t*)blk;
        r.v[0] = __ldg(b16 + (64 * h + l0) / 2);              // ql[l0], ql[l0+1]
        r.v[1] = __ldg(b16 + (64 * h + 32 + l0) / 2);         // ql[l0+32], ql[l0+33]
        r.v[2] = __ldg(b16 + (128 + 32 * h + l0) / 2);        // qh[l0], qh[l0+1]
        r.v[3] = __ldg(b16 + (192 + 8 * h) / 2) | ((uint32_t)__ldg(b16 + (194 + 8 * h) / 2) << 16);
        r.v[4] = __ldg(b16 + (196 + 8 * h) / 2) | ((uint32_t)__ldg(b16 + (198 + 8 * h) / 2) << 16);
        r.v[5] = __ldg(b16 + 104);                            // d
    } else {
        constexpr bool five = T == CW_GGUF_Q5_K;
        const uint32_t* b32 = (const uint32_t*)blk;
        const int c = lane >> 3, j = lane & 7;
        r.v[0] = __ldg(b32 + 0);  // d, dmin
        r.v[1] = __ldg(b32 + 1);  // scales 0..3
        r.v[2] = __ldg(b32 + 2);  // scales 4..7
        r.v[3] = __ldg(b32 + 3);  // scales 8..11
        r.v[4] = __ldg(b32 + (five ? 12 : 4) + 8 * c + j);  // 4 nibble bytes
        r.v[5] = five ? __ldg(b32 + 4 + j) : 0u;            // 4 fifth-bit bytes
    }
    return r;
}

__device__ __forceinline__ float kq_h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xffffu)));
}

// Partial dot of one lane's 8 weights of a block with x (xb = block's x).
template <int T>
__device__ __forceinline__ float kq_dot(const KqRaw<T>& r, const float* __restrict__ xb, int lane,
                                        float acc) {
    if constexpr (kq_consecutive<T>()) {
        const float4 x0 = *reinterpret_cast<const float4*>(xb + 8 * lane);
        const float4 x1 = *reinterpret_cast<const float4*>(xb + 8 * lane + 4);
        const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        if constexpr (T == CW_GGUF_Q8_0) {  // d * sum(q x)
            float s = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++)
                s = fmaf((float)(int8_t)((r.v[i >> 2] >> (8 * (i & 3))) & 0xff), x[i], s);
            return fmaf(kq_h2f(r.v[2]), s, acc);
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                float w;
                if constexpr (T == CW_GGUF_F32) w = __uint_as_float(r.v[i]);
                else if constexpr (T == CW_GGUF_F16) w = kq_h2f(r.v[i >> 1] >> (16 * (i & 1)));
                else w = kq_bf16(r.v[i >> 1] >> (16 * (i & 1)));
                acc = fmaf(w, x[i], acc);
            }
            return acc;
        }
    } else if constexpr (T == CW_GGUF_Q4_1) {  // d * sum(q x) + m * sum(x)
        const int c = lane >> 2, j0 = 4 * (lane & 3);
        const float4 xl = *reinterpret_cast<const float4*>(xb + 32 * c + j0);
        const float4 xh = *reinterpret_cast<const float4*>(xb + 32 * c + 16 + j0);
        const uint32_t q = r.v[1];
        float s = (float)(q & 0x0f) * xl.x;
        s = fmaf((float)((q >> 8) & 0x0f), xl.y, s);
        s = fmaf((float)((q >> 16) & 0x0f), xl.z, s);
        s = fmaf((float)((q >> 24) & 0x0f), xl.w, s);
        s = fmaf((float)((q >> 4) & 0x0f), xh.x, s);
        s = fmaf((float)((q >> 12) & 0x0f), xh.y, s);
        s = fmaf((float)((q >> 20) & 0x0f), xh.z, s);
        s = fmaf((float)(q >> 28), xh.w, s);
        const float sx = ((xl.x + xl.y) + (xl.z + xl.w)) + ((xh.x + xh.y) + (xh.z + xh.w));
        acc = fmaf(kq_h2f(r.v[0]), s, acc);
        return fmaf(kq_h2f(r.v[0] >> 16), sx, acc);
    } else if constexpr (T == CW_GGUF_Q6_K) {
        const int h = lane >> 4, l0 = 2 * (lane & 15), is = l0 >> 4;
        const float d = kq_h2f(r.v[5]);
        const uint32_t scw = is ? (r.v[3] >> 8) | (r.v[4] << 24) : r.v[3];  // sc[is..is+3]
        const uint32_t scw2 = is ? (r.v[4] >> 8) : r.v[4];                 // sc[is+4..]
        const float s0 = (float)(int8_t)(scw & 0xff), s2 = (float)(int8_t)((scw >> 16) & 0xff);
        const float s4 = (float)(int8_t)(scw2 & 0xff), s6 = (float)(int8_t)((scw2 >> 16) & 0xff);
        const float ds0 = __fmul_rn(d, s0), ds2 = __fmul_rn(d, s2);
        const float ds4 = __fmul_rn(d, s4), ds6 = __fmul_rn(d, s6);
        // per scale, the two weights' q*x first, then one multiply by d*sc
        float t1 = 0.f, t2 = 0.f, t3 = 0.f, t4 = 0.f;
        const float* xl = xb + 128 * h + l0;
        const float2 x1 = *reinterpret_cast<const float2*>(xl);
        const float2 x2 = *reinterpret_cast<const float2*>(xl + 32);
        const float2 x3 = *reinterpret_cast<const float2*>(xl + 64);
        const float2 x4 = *reinterpret_cast<const float2*>(xl + 96);
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int a = (r.v[0] >> (8 * u)) & 0xff, b = (r.v[1] >> (8 * u)) & 0xff;
            const int hb = (r.v[2] >> (8 * u)) & 0xff;
            const int q1 = ((a & 0x0f) | ((hb & 3) << 4)) - 32;
            const int q2 = ((b & 0x0f) | (((hb >> 2) & 3) << 4)) - 32;
            const int q3 = ((a >> 4) | (((hb >> 4) & 3) << 4)) - 32;
            const int q4 = ((b >> 4) | (((hb >> 6) & 3) << 4)) - 32;
            t1 = fmaf((float)q1, u ? x1.y : x1.x, t1);
            t2 = fmaf((float)q2, u ? x2.y : x2.x, t2);
            t3 = fmaf((float)q3, u ? x3.y : x3.x, t3);
            t4 = fmaf((float)q4, u ? x4.y : x4.x, t4);
        }
        acc = fmaf(ds0, t1, acc);
        acc = fmaf(ds2, t2, acc);
        acc = fmaf(ds4, t3, acc);
        acc = fmaf(ds6, t4, acc);
        return acc;
    } else {
        // lane j (of each 8) decodes (scale, min) pair j; lane l then takes
        // pairs 2c, 2c+1 (c = l/8) by shuffle.  The sub-block sum is
        // d1 * sum(q x) - dmin*m * sum(x), sum(x) per 4 x values from xs4.
        constexpr bool five = T == CW_GGUF_Q5_K;
        const int c = lane >> 3, j0 = 4 * (lane & 7), jp = lane & 7;
        const float d = kq_h2f(r.v[0]), dmin = kq_h2f(r.v[0] >> 16);
        const uint32_t sw[3] = {r.v[1], r.v[2], r.v[3]};
        auto byte = [&](int i) { return (int)((sw[i >> 2] >> (8 * (i & 3))) & 0xff); };
        int sc, m;
        if (jp < 4) {
            sc = byte(jp) & 63;
            m = byte(jp + 4) & 63;
        } else {
            sc = (byte(jp + 4) & 0x0f) | ((byte(jp - 4) >> 6) << 4);
            m = (byte(jp + 4) >> 4) | ((byte(jp) >> 6) << 4);
        }
        const float ds = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)m);
        const float d1 = __shfl_sync(0xffffffffu, ds, 2 * c), mm1 = __shfl_sync(0xffffffffu, dm, 2 * c);
        const float d2 = __shfl_sync(0xffffffffu, ds, 2 * c + 1),
                    mm2 = __shfl_sync(0xffffffffu, dm, 2 * c + 1);
        const float* x0 = xb + 64 * c + j0;
        const float4 xl = *reinterpret_cast<const float4*>(x0);
        const float4 xh = *reinterpret_cast<const float4*>(x0 + 32);
        const uint32_t qw = r.v[4];
        uint32_t lo4 = qw & 0x0f0f0f0fu, hi4 = (qw >> 4) & 0x0f0f0f0fu;
        if constexpr (five) {
            const uint32_t hb = r.v[5];
            lo4 |= ((hb >> (2 * c)) & 0x01010101u) << 4;
            hi4 |= ((hb >> (2 * c + 1)) & 0x01010101u) << 4;
        }
        float ql = (float)(lo4 & 0xff) * xl.x;
        ql = fmaf((float)((lo4 >> 8) & 0xff), xl.y, ql);
        ql = fmaf((float)((lo4 >> 16) & 0xff), xl.z, ql);
        ql = fmaf((float)(lo4 >> 24), xl.w, ql);
        float qhs = (float)(hi4 & 0xff) * xh.x;
        qhs = fmaf((float)((hi4 >> 8) & 0xff), xh.y, qhs);
        qhs = fmaf((float)((hi4 >> 16) & 0xff), xh.z, qhs);
        qhs = fmaf((float)(hi4 >> 24), xh.w, qhs);
        const float sxl = (xl.x + xl.y) + (xl.z + xl.w), sxh = (xh.x + xh.y) + (xh.z + xh.w);
        acc = fmaf(d1, ql, acc);
        acc = fmaf(-mm1, sxl, acc);
        acc = fmaf(d2, qhs, acc);
        acc = fmaf(-mm2, sxh, acc);
        return acc;
    }
}

constexpr int KQ_UNROLL = 4;  // super-blocks whose loads are in flight together


// Element j (0..255) of a Q6_K super-block (dequant.rs:113-128 for one index).
__device__ __forceinline__ float q6k_elem(const uint8_t* __restrict__ blk, int j) {
    const int h = j >> 7, l = j & 127, quad = l >> 5, ll = l & 31, is = ll >> 4;
    const int qlb = blk[64 * h + ll + ((quad & 1) ? 32 : 0)];
    const int qhb = blk[128 + 32 * h + ll];
    const int q = (((quad >= 2) ? (qlb >> 4) : (qlb & 0x0f)) | (((qhb >> (2 * quad)) & 3) << 4)) - 32;
    const float d = kq_f16(blk + 208);
    const float sc = (float)(int8_t)blk[192 + 8 * h + is + 2 * quad];
    return __fmul_rn(__fmul_rn(d, sc), (float)q);
}

// Weight j (0..255) of a Q4_K / Q5_K super-block: chunk c = j / 64, its low
// nibbles (scale/min pair 2c) for j % 64 < 32, else its high nibbles (pair
// 2c+1); w = (d*sc)*q - dmin*m, the rounding steps of kq_lane.
template <bool FIVE>
__device__ __forceinline__ float q45k_elem(const uint8_t* __restrict__ blk, int j) {
    const int c = j >> 6, l = j & 31, hi = (j >> 5) & 1;
    int sc, m;
    kq_scale_min(2 * c + hi, blk + 4, &sc, &m);
    const int qb = blk[(FIVE ? 48 : 16) + 32 * c + l];
    int q = hi ? (qb >> 4) : (qb & 0x0f);
    if (FIVE) q += ((blk[16 + l] >> (2 * c + hi)) & 1) << 4;
    const float d1 = __fmul_rn(kq_f16(blk), (float)sc), mm = __fmul_rn(kq_f16(blk + 2), (float)m);
    return __fsub_rn(__fmul_rn(d1, (float)q), mm);
}

// Element i of row `tok` of a token-embedding table: packed Q4_0 planes
// (type 2, dequant.rs:62-78) or the file's raw rows of any other type the
// loader keeps raw (dim % 256 == 0).
__device__ __forceinline__ float embed_elem(const uint8_t* __restrict__ payload,
                                            const __half* __restrict__ scales, int type,
                                            unsigned tok, int dim, int i) {
    const size_t e = (size_t)tok * dim + i;
    if (type == CW_GGUF_F32) return reinterpret_cast<const float*>(payload)[e];
    if (type == CW_GGUF_F16) return kq_f16(payload + 2 * e);
    if (type == CW_GGUF_BF16) return kq_bf16(reinterpret_cast<const uint16_t*>(payload)[e]);
    if (type == CW_GGUF_Q8_0) {  // dequant.rs:46-58
        const uint8_t* b = payload + (e >> 5) * 34;
        return __fmul_rn(kq_f16(b), (float)(int8_t)b[2 + (i & 31)]);
    }
    if (type == CW_GGUF_Q4_1) {  // dequant.rs:82-97
        const uint8_t* b = payload + (e >> 5) * 20;
        const int j = i & 31, byte = b[4 + (j & 15)];
        const int q = j < 16 ? (byte & 0x0f) : (byte >> 4);
        return __fadd_rn(__fmul_rn(kq_f16(b), (float)q), kq_f16(b + 2));
    }
    if (type == CW_GGUF_Q6_K)
        return q6k_elem(payload + ((size_t)tok * (dim / 256) + (i >> 8)) * 210, i & 255);
    if (type == CW_GGUF_Q4_K)
        return q45k_elem<false>(payload + ((size_t)tok * (dim / 256) + (i >> 8)) * 144, i & 255);
    if (type == CW_GGUF_Q5_K)
        return q45k_elem<true>(payload + ((size_t)tok * (dim / 256) + (i >> 8)) * 176, i & 255);
    const int nb = dim / 32, b = i >> 5, j = i & 31;
    const size_t blk = (size_t)tok * nb + b;
    const float d = __half2float(scales[blk]);
    const uint8_t byte = payload[blk * 16 + (j & 15)];
    const int q = (j < 16) ? (byte & 0xf) : (byte >> 4);
    return __fmul_rn(d, (float)(q - 8));
}

// Split nsb raw Q6_K super-blocks (210 bytes each) into the streaming GEMV's
// aligned planes: pay [nsb][208] (ql, qh, scales) and d [nsb] (f16).
int q6k_split(cw_ctx* ctx, const uint8_t* raw, size_t nsb, uint8_t* pay, __half* d);
// Split nb raw Q8_0 blocks (34 bytes: f16 d, 32 int8 codes) into the codes
// plane pay [nb][32] and the scales d [nb].
int q8_split(cw_ctx* ctx, const uint8_t* raw, size_t nb, uint8_t* pay, __half* d);

}  // namespace cw
