// cw_prefill.cu -- batched prompt prefill: the prompt's rows go through each
// layer together, with every projection on the tcgen05 tensor cores
// (cw_gemm.cuh) instead of one Q4 GEMV per token.
//
// The reference runs the prompt one token at a time (src/model/mod.rs:78-83)
// through the same layer composition as decode (src/model/qwen3.rs:139-191).
// Prefill reproduces that composition over C rows at positions p0 .. p0+C-1:
//
//   embed      H[r]   = dequant(token_embd[prompt[p0+r]])          (qwen3.rs:128-133)
//   per layer
//     norm     X      = rmsnorm(H) (+ post-norm residual, gemma2)  (norm.wgsl:20-56)
//     qkv      QKV    = X Wqkv^T (+bias)                            tcgen05 GEMM
//     qk       QK-norm, RoPE at the row's position; K, V rows into the cache
//     attn     causal attention of each row over cache positions <= its own
//     o        H     += O Wo^T            (gemma2: T = O Wo^T, added post-normed)
//     norm, gate/up GEMM, SwiGLU/GeGLU, down GEMM the same way
//
// The last layer stops after writing K and V: no later computation reads the
// prefill rows' hidden states, because the final prompt token runs through
// the decode step, which produces the first token's logits exactly as the
// token-by-token loop does.  Activations feed the GEMMs as f16 hi/lo pairs
// (cw_gemm.cuh); each weight matrix is split into its f16 pair once per
// chunk, into a session scratch reused across layers.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <memory>

#include "cw_attn.cuh"
#include "cw_common.h"
#include "cw_device.cuh"
#include "cw_gemm.cuh"
#include "cw_gemv.cuh"
#include "cw_mgemv.h"
#include "cw_kquant.cuh"
#include "cw_model.h"
#include "cw_sample.cuh"

namespace cw {

constexpr int PF_CHUNK = 4096;  // rows per prefill chunk (bounds the scratch)

__device__ __forceinline__ float pf_block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

// Rows of token_embd for prompt[0 .. C), exact dequantisation (Q4_0 or Q6_K).
__global__ void k_pf_embed(const uint8_t* __restrict__ payload, const __half* __restrict__ scales,
                           int type, int dim, float scale, const unsigned* __restrict__ toks,
                           float* __restrict__ H) {
    const int r = blockIdx.x;
    const unsigned tok = toks[r];
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = embed_elem(payload, scales, type, tok, dim, i);
        H[(size_t)r * dim + i] = scale > 0.f ? __fmul_rn(v, scale) : v;
    }
}

// Row r: h = H[r] (+ rmsnorm(T[r]) * gain(post_w), written back to H), then
// X = rmsnorm(h) * gain(norm_w) as an f16 hi/lo pair.
__global__ void __launch_bounds__(256) k_pf_norm(float* __restrict__ H, const float* __restrict__ T,
                                                 const float* __restrict__ post_w,
                                                 const float* __restrict__ norm_w, int unit,
                                                 float eps, int dim, __half* __restrict__ xh,
                                                 __half* __restrict__ xl) {
    pdl_trigger();
    pdl_wait();
    extern __shared__ float hb[];
    __shared__ float red[32];
    const size_t r0 = (size_t)blockIdx.x * dim;
    float inv_d = 0.f;
    if (T && post_w) {
        float ss = 0.f;
        for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(T[r0 + i], T[r0 + i], ss);
        ss = pf_block_sum(ss, red);
        inv_d = 1.0f / sqrtf(ss / (float)dim + eps);
    }
    float ssh = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float h = H[r0 + i];
        if (T) {
            float dv = T[r0 + i];
            if (post_w) {
                const float gw = unit ? 1.0f + post_w[i] : post_w[i];
                dv = __fmul_rn(__fmul_rn(dv, inv_d), gw);
            }
            h = h + dv;
            H[r0 + i] = h;
        }
        hb[i] = h;
        ssh = fmaf(h, h, ssh);
    }
    if (!xh) return;  // residual update only
    ssh = pf_block_sum(ssh, red);
    const float inv = 1.0f / sqrtf(ssh / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float g = unit ? 1.0f + norm_w[i] : norm_w[i];
        split_f16(__fmul_rn(__fmul_rn(hb[i], inv), g), xh + r0 + i, xl + r0 + i);
    }
}

// Row r, one warp per head: QK-norm (qwen3.rs:154-155), RoPE at position
// p0 + r (rope.wgsl:25-34); q back in place, k and v into the cache
// (cache.rs:21-24, layout [n_kv][max_seq][hd]).
__global__ void __launch_bounds__(256) k_pf_qk(float* __restrict__ QKV, int ld,
                                               const float* __restrict__ q_norm,
                                               const float* __restrict__ k_norm, float eps,
                                               const float* __restrict__ inv_freq,
                                               float* __restrict__ kc, float* __restrict__ vc,
                                               int max_seq, int p0, int nh, int nkv, int hd) {
    extern __shared__ float rb[];
    const int r = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nw = blockDim.x >> 5, pos = p0 + r, half = hd / 2;
    const int qd = nh * hd, kvd = nkv * hd;
    float* row = QKV + (size_t)r * ld;
    float* sb = rb + (size_t)warp * hd;
    for (int h = warp; h < nh + nkv; h += nw) {
        const bool isq = h < nh;
        float* src = isq ? row + (size_t)h * hd : row + qd + (size_t)(h - nh) * hd;
        const float* nwt = isq ? q_norm : k_norm;
        float ss = 0.f;
        for (int d = lane; d < hd; d += 32) {
            const float v = src[d];
            sb[d] = v;
            ss = fmaf(v, v, ss);
        }
        __syncwarp();
        if (nwt) {
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
            for (int d = lane; d < hd; d += 32) sb[d] = __fmul_rn(__fmul_rn(sb[d], inv), nwt[d]);
            __syncwarp();
        }
        float* dst = isq ? src : kc + ((size_t)(h - nh) * max_seq + pos) * hd;
        for (int k = lane; k < half; k += 32) {
            const float freq = __fmul_rn((float)pos, inv_freq[k]);
            float sn, cs;
            sincosf(freq, &sn, &cs);
            const float lo = sb[k], hi = sb[k + half];
            dst[k] = __fsub_rn(__fmul_rn(lo, cs), __fmul_rn(hi, sn));
            dst[k + half] = __fadd_rn(__fmul_rn(hi, cs), __fmul_rn(lo, sn));
        }
        __syncwarp();
    }
    for (int i = threadIdx.x; i < kvd; i += blockDim.x) {
        const int g = i / hd, d = i - g * hd;
        vc[((size_t)g * max_seq + pos) * hd + d] = row[qd + kvd + i];
    }
}

// Row r, kv head g: the G query heads of the group attend over cache
// positions [j0, p0 + r] (attention.wgsl:33-95 via attn_core; sliding window
// and soft-cap as in decode); the output goes out as an f16 hi/lo pair.
template <int EPL, int GMAX>
__global__ void __launch_bounds__(128) k_pf_attn(const float* __restrict__ QKV, int ld,
                                                 const float* __restrict__ kc,
                                                 const float* __restrict__ vc, int max_seq, int p0,
                                                 int nh, int nkv, int hd, int window, float scale,
                                                 float softcap, __half* __restrict__ xh,
                                                 __half* __restrict__ xl) {
    extern __shared__ float sm[];
    const int r = blockIdx.x, g = blockIdx.y, G = nh / nkv, W = hd + 2;
    const int seq = p0 + r + 1;
    float* qs = sm + attn_smem_floats(G, hd, 1);
    const float* qsrc = QKV + (size_t)r * ld + (size_t)g * G * hd;
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i] = qsrc[i];
    __syncthreads();
    int jlo, jhi;
    attn_range(seq, window, 0, 1, &jlo, &jhi);
    float* res = sm + 4 * G * W;
    attn_core<EPL, GMAX, KV_NC>(qs, G, hd, kc + (size_t)g * max_seq * hd,
                                vc + (size_t)g * max_seq * hd, hd, jlo, jhi, scale, softcap, sm,
                                res);
    const size_t o0 = (size_t)r * nh * hd + (size_t)g * G * hd;
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int gi = i / hd, d = i - gi * hd;
        const float o = res[gi * W + d] * (1.0f / res[gi * W + hd + 1]);
        split_f16(o, xh + o0 + i, xl + o0 + i);
    }
}

// Tiled causal attention for head_dim HD in {64, 128, 256}: a CTA takes 64
// consecutive query rows of one head and streams the kv head's cache rows
// through shared memory 32 keys at a time, so every K/V row read serves 64
// queries (k_pf_attn above re-reads them per query).  Same f32 arithmetic
// as the decode path (attention.wgsl:33-95): scores q.k * scale (soft-capped),
// an online softmax per query row with running max and denominator, keys
// limited to [pos - window + 1, pos] on windowed layers.
// Thread (tr, tc) = (tid / 16, tid % 16) owns query rows tr + 16i (i < 4),
// score columns tc + 16j (j < 2) and output dims 4tc + 64jj .. +3; the 16
// threads of a row form a half-warp, which reduces the row max and sum.
constexpr int PFA_BQ = 64, PFA_BK = 32;

__host__ __device__ constexpr size_t pfa_smem(int hd) {
    return ((size_t)PFA_BQ * (hd + 4) + (size_t)PFA_BK * (hd + 4) + (size_t)PFA_BK * hd +
            (size_t)PFA_BQ * (PFA_BK + 1)) *
           sizeof(float);
}

__device__ __forceinline__ float hw_max(float v) {  // over the 16 lanes of a half-warp
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
    return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
}
__device__ __forceinline__ float hw_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 8);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v + __shfl_xor_sync(0xffffffffu, v, 1);
}

template <int HD>
__global__ void __launch_bounds__(256) k_pf_fattn(const float* __restrict__ QKV, int ld,
                                                  const float* __restrict__ kc,
                                                  const float* __restrict__ vc, int max_seq,
                                                  int p0, int C, int nh, int nkv, int window,
                                                  float scale, float softcap,
                                                  __half* __restrict__ xh,
                                                  __half* __restrict__ xl) {
    constexpr int BQ = PFA_BQ, BK = PFA_BK, QS = HD + 4, NJ = HD / 64, PS = BK + 1;
    extern __shared__ __align__(16) float pfa[];
    float* Qs = pfa;             // [BQ][QS]
    float* Ks = Qs + BQ * QS;    // [BK][QS]
    float* Vs = Ks + BK * QS;    // [BK][HD]
    float* Ps = Vs + BK * HD;    // [BQ][PS]
    const int tid = threadIdx.x, tr = tid >> 4, tc = tid & 15;
    // longest rows (latest positions) first: the causal work grows with the row
    const int r0 = (gridDim.x - 1 - blockIdx.x) * BQ;
    const int h = blockIdx.y, g = h / (nh / nkv);
    const int nrows = min(BQ, C - r0);
    for (int i = tid; i < BQ * (HD / 4); i += blockDim.x) {
        const int r = i / (HD / 4), c4 = i - r * (HD / 4);
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nrows) v = *reinterpret_cast<const float4*>(QKV + (size_t)(r0 + r) * ld +
                                                            (size_t)h * HD + 4 * c4);
        *reinterpret_cast<float4*>(Qs + r * QS + 4 * c4) = v;
    }
    const int pos_first = p0 + r0, j_end = p0 + r0 + nrows;  // keys [j_begin, j_end)
    const int j_begin = window > 0 ? max(0, pos_first - window + 1) : 0;
    int pos[4];
    float m[4], l[4];
    float4 acc[4][NJ];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        pos[i] = pos_first + tr + 16 * i;
        m[i] = REF_NEG_INF;
        l[i] = 0.f;
#pragma unroll
        for (int jj = 0; jj < NJ; jj++) acc[i][jj] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float* kb = kc + (size_t)g * max_seq * HD;
    const float* vb = vc + (size_t)g * max_seq * HD;
    for (int kt = j_begin; kt < j_end; kt += BK) {
        __syncthreads();  // previous tile's K, V, P consumed (and Q stored, first time)
        for (int i = tid; i < BK * (HD / 4); i += blockDim.x) {
            const int r = i / (HD / 4), c4 = i - r * (HD / 4);
            float4 kv = make_float4(0.f, 0.f, 0.f, 0.f), vv = kv;
            if (kt + r < j_end) {
                kv = __ldg(reinterpret_cast<const float4*>(kb + (size_t)(kt + r) * HD) + c4);
                vv = __ldg(reinterpret_cast<const float4*>(vb + (size_t)(kt + r) * HD) + c4);
            }
            *reinterpret_cast<float4*>(Ks + r * QS + 4 * c4) = kv;
            *reinterpret_cast<float4*>(Vs + r * HD + 4 * c4) = vv;
        }
        __syncthreads();
        float s[4][2];
#pragma unroll
        for (int i = 0; i < 4; i++) s[i][0] = s[i][1] = 0.f;
#pragma unroll 4
        for (int d = 0; d < HD; d += 4) {
            float4 k4[2], q4[4];
#pragma unroll
            for (int j = 0; j < 2; j++)
                k4[j] = *reinterpret_cast<const float4*>(Ks + (tc + 16 * j) * QS + d);
#pragma unroll
            for (int i = 0; i < 4; i++)
                q4[i] = *reinterpret_cast<const float4*>(Qs + (tr + 16 * i) * QS + d);
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 2; j++) {
                    float t = s[i][j];
                    t = fmaf(q4[i].x, k4[j].x, t);
                    t = fmaf(q4[i].y, k4[j].y, t);
                    t = fmaf(q4[i].z, k4[j].z, t);
                    t = fmaf(q4[i].w, k4[j].w, t);
                    s[i][j] = t;
                }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float mx = REF_NEG_INF;
            bool ok[2];
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int key = kt + tc + 16 * j;
                ok[j] = key <= pos[i] && key < j_end && (window <= 0 || key > pos[i] - window);
                float v = s[i][j] * scale;
                if (softcap > 0.f) v = softcap * tanhf(v / softcap);
                s[i][j] = v;
                if (ok[j]) mx = fmaxf(mx, v);
            }
            mx = hw_max(mx);
            const float mn = fmaxf(m[i], mx);
            const float corr = expf(m[i] - mn);
            float ps = 0.f;
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const float p = ok[j] ? expf(s[i][j] - mn) : 0.f;
                Ps[(tr + 16 * i) * PS + tc + 16 * j] = p;
                ps += p;
            }
            l[i] = l[i] * corr + hw_sum(ps);
            m[i] = mn;
#pragma unroll
            for (int jj = 0; jj < NJ; jj++) {
                acc[i][jj].x *= corr;
                acc[i][jj].y *= corr;
                acc[i][jj].z *= corr;
                acc[i][jj].w *= corr;
            }
        }
        __syncthreads();
#pragma unroll 4
        for (int c = 0; c < BK; c++) {
            float p[4];
#pragma unroll
            for (int i = 0; i < 4; i++) p[i] = Ps[(tr + 16 * i) * PS + c];
#pragma unroll
            for (int jj = 0; jj < NJ; jj++) {
                const float4 v = *reinterpret_cast<const float4*>(Vs + c * HD + 4 * tc + 64 * jj);
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    acc[i][jj].x = fmaf(v.x, p[i], acc[i][jj].x);
                    acc[i][jj].y = fmaf(v.y, p[i], acc[i][jj].y);
                    acc[i][jj].z = fmaf(v.z, p[i], acc[i][jj].z);
                    acc[i][jj].w = fmaf(v.w, p[i], acc[i][jj].w);
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int r = tr + 16 * i;
        if (r >= nrows) continue;
        const float inv = 1.0f / l[i];
        const size_t o = (size_t)(r0 + r) * nh * HD + (size_t)h * HD + 4 * tc;
#pragma unroll
        for (int jj = 0; jj < NJ; jj++) {
            const size_t oj = o + 64 * jj;
            split_f16(acc[i][jj].x * inv, xh + oj + 0, xl + oj + 0);
            split_f16(acc[i][jj].y * inv, xh + oj + 1, xl + oj + 1);
            split_f16(acc[i][jj].z * inv, xh + oj + 2, xl + oj + 2);
            split_f16(acc[i][jj].w * inv, xh + oj + 3, xl + oj + 3);
        }
    }
}

// ---- causal prefill attention on the tensor cores (head_dim 128) ----------------
// The same attention as k_pf_fattn (online softmax per query row, the
// attention.wgsl merge rule) with both products on the warp-level f16 MMA
// (mma.sync m16n8k16, f32 accumulation).  f16 alone misses the 1e-3 gate, so
// every operand is split into an f16 pair x = xh + xl (xl = f16(x - xh),
// ~22 bits together) and each product takes three MMAs, hh + hl + lh (the
// dropped ll term is 2^-22 relative): S = QK^T from the Q and K pairs, then
// O += P V from the probabilities P (split in registers straight from the S
// accumulators: the m16n8 C layout of two key tiles is the m16n8k16 A layout)
// and the V pair.  The layer's K and V rows are split into pairs once
// (k_pf_kv_pairs); a CTA takes 64 query rows of one head (4 warps of 16 rows)
// and streams its kv head's pairs 32 keys at a time with cp.async into two
// shared-memory buffers, the next tile landing while the current one is
// multiplied (rows padded by 16 bytes: the ldmatrix row addresses of a
// fragment fall in distinct banks).  No soft-cap or window (those layers keep
// k_pf_fattn).
constexpr int PTC_BQ = 64, PTC_BK = 32, PTC_HD = 128, PTC_P = PTC_HD + 8;  // row pitch, halves
constexpr size_t PTC_SMEM = ((size_t)2 * PTC_BQ + (size_t)2 * 4 * PTC_BK) * PTC_P * sizeof(__half);

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const __half* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const __half* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2_bits(__half2 v) { return *reinterpret_cast<uint32_t*>(&v); }
// f32 pair -> (hi, lo) f16 pairs
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    hi = h2_bits(h);
    lo = h2_bits(__floats2half2_rn(a - hf.x, b - hf.y));
}
// four f32 -> hi / lo f16 stores (8-byte aligned)
__device__ __forceinline__ void split_store4(const float4& v, __half* hi, __half* lo) {
    uint32_t h0, l0, h1, l1;
    split_h2(v.x, v.y, h0, l0);
    split_h2(v.z, v.w, h1, l1);
    *reinterpret_cast<uint2*>(hi) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(lo) = make_uint2(l0, l1);
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}

// The K and V cache rows [0, n) of one layer (all kv heads, [kv][max_seq][128]
// f32) as f16 pairs kp = [Kh | Kl | Vh | Vl], each [kv][stride][128]; rows
// [n, n_pad) are zeros, so a key tile past the live keys multiplies finite
// values (masked to zero weight).
__global__ void k_pf_kv_pairs(const float* __restrict__ kc, const float* __restrict__ vc,
                              int max_seq, int nkv, int n, int n_pad, int stride,
                              __half* __restrict__ kp) {
    pdl_trigger();
    pdl_wait();
    const size_t plane = (size_t)nkv * stride * PTC_HD;
    const long total = (long)nkv * n_pad * (PTC_HD / 4);
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total;
         i += (long)gridDim.x * blockDim.x) {
        const int g = (int)(i / ((long)n_pad * (PTC_HD / 4)));
        const long rem = i - (long)g * n_pad * (PTC_HD / 4);
        const int r = (int)(rem / (PTC_HD / 4)), c4 = (int)(rem % (PTC_HD / 4));
        float4 k = make_float4(0.f, 0.f, 0.f, 0.f), v = k;
        if (r < n) {
            k = *reinterpret_cast<const float4*>(kc + ((size_t)g * max_seq + r) * PTC_HD + 4 * c4);
            v = *reinterpret_cast<const float4*>(vc + ((size_t)g * max_seq + r) * PTC_HD + 4 * c4);
        }
        const size_t o = ((size_t)g * stride + r) * PTC_HD + 4 * c4;
        split_store4(k, kp + o, kp + plane + o);
        split_store4(v, kp + 2 * plane + o, kp + 3 * plane + o);
    }
}

__global__ void __launch_bounds__(128) k_pf_attn_tc(const float* __restrict__ QKV, int ld,
                                                    const __half* __restrict__ kp, int stride,
                                                    int p0, int C, int nh, int nkv, float scale,
                                                    __half* __restrict__ xh,
                                                    __half* __restrict__ xl) {
    pdl_trigger();
    extern __shared__ __align__(16) __half ptc[];
    __half* Qh = ptc;
    __half* Ql = Qh + PTC_BQ * PTC_P;
    __half* KV = Ql + PTC_BQ * PTC_P;  // [2 buffers][Kh, Kl, Vh, Vl][32][PTC_P]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, c = lane & 3;
    // longest rows (latest positions) first: the causal work grows with the row
    const int r0 = (gridDim.x - 1 - blockIdx.x) * PTC_BQ;
    const int h = blockIdx.y, kvh = h / (nh / nkv);
    const int nrows = min(PTC_BQ, C - r0);
    const size_t plane = (size_t)nkv * stride * PTC_HD;
    const __half* src0 = kp + (size_t)kvh * stride * PTC_HD;
    const int pos_first = p0 + r0, j_end = p0 + r0 + nrows;  // keys [0, j_end)
    const int n_tiles = (j_end + PTC_BK - 1) / PTC_BK;
    // tile t of the kv head's pairs into buffer t % 2 (16 cp.async per thread)
    auto load_tile = [&](int t) {
        __half* dst = KV + (size_t)(t & 1) * 4 * PTC_BK * PTC_P;
        for (int i = tid; i < 4 * PTC_BK * 16; i += 128) {
            const int mat = i >> 9, r = (i >> 4) & (PTC_BK - 1), ch = i & 15;
            cp_async16(dst + ((size_t)mat * PTC_BK + r) * PTC_P + 8 * ch,
                       src0 + mat * plane + (size_t)(t * PTC_BK + r) * PTC_HD + 8 * ch);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    pdl_wait();
    load_tile(0);
    for (int i = tid; i < PTC_BQ * 32; i += 128) {  // Q rows (normed, roped) -> f16 pairs
        const int r = i >> 5, c4 = i & 31;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (r < nrows)
            v = *reinterpret_cast<const float4*>(QKV + (size_t)(r0 + r) * ld + (size_t)h * PTC_HD + 4 * c4);
        split_store4(v, Qh + r * PTC_P + 4 * c4, Ql + r * PTC_P + 4 * c4);
    }
    const int rw = warp * 16;  // this warp's first row
    const int pos_g = pos_first + rw + g, pos_g8 = pos_g + 8;
    float o[16][4];
#pragma unroll
    for (int n = 0; n < 16; n++) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = REF_NEG_INF, m1 = REF_NEG_INF, l0 = 0.f, l1 = 0.f;
    // ldmatrix row addresses (thread t: matrix t / 8, row t % 8)
    const int lrow = (lane & 7) + 8 * ((lane >> 3) & 1), lcol = 8 * (lane >> 4);
    for (int t = 0; t < n_tiles; t++) {
        if (t + 1 < n_tiles) {
            load_tile(t + 1);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();  // tile t (and, the first time, Q) visible to every warp
        const __half* Kh = KV + (size_t)(t & 1) * 4 * PTC_BK * PTC_P;
        const __half* Kl = Kh + PTC_BK * PTC_P;
        const __half* Vh = Kl + PTC_BK * PTC_P;
        const __half* Vl = Vh + PTC_BK * PTC_P;
        const int kt = t * PTC_BK;
        // ---- S = Q K^T over the tile: 4 key tiles of 8, hd in 8 steps of 16
        float sacc[4][4];
#pragma unroll
        for (int n = 0; n < 4; n++) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            uint32_t qh[4], ql[4];
            ldsm_x4(qh, Qh + (rw + lrow) * PTC_P + ks * 16 + lcol);
            ldsm_x4(ql, Ql + (rw + lrow) * PTC_P + ks * 16 + lcol);
#pragma unroll
            for (int np = 0; np < 2; np++) {
                // keys np*16 + (t%8) + 8*(t/16), hd ks*16 + 8*((t/8)%2): matrices
                // (key tile 2np: b0, b1), (key tile 2np+1: b0, b1)
                const int krow = np * 16 + (lane & 7) + 8 * (lane >> 4), kcol = ks * 16 + 8 * ((lane >> 3) & 1);
                uint32_t khf[4], klf[4];
                ldsm_x4(khf, Kh + krow * PTC_P + kcol);
                ldsm_x4(klf, Kl + krow * PTC_P + kcol);
                mma_f16(sacc[2 * np], qh, khf[0], khf[1]);
                mma_f16(sacc[2 * np], qh, klf[0], klf[1]);
                mma_f16(sacc[2 * np], ql, khf[0], khf[1]);
                mma_f16(sacc[2 * np + 1], qh, khf[2], khf[3]);
                mma_f16(sacc[2 * np + 1], qh, klf[2], klf[3]);
                mma_f16(sacc[2 * np + 1], ql, khf[2], khf[3]);
            }
        }
        // ---- online softmax: this thread's rows g and g + 8, keys 8n + 2c, +1
        float mx0 = REF_NEG_INF, mx1 = REF_NEG_INF;
#pragma unroll
        for (int n = 0; n < 4; n++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int key = kt + 8 * n + 2 * c + e;
                const float v0 = sacc[n][e] * scale, v1 = sacc[n][2 + e] * scale;
                sacc[n][e] = key <= pos_g && key < j_end ? v0 : REF_NEG_INF;
                sacc[n][2 + e] = key <= pos_g8 && key < j_end ? v1 : REF_NEG_INF;
                mx0 = fmaxf(mx0, sacc[n][e]);
                mx1 = fmaxf(mx1, sacc[n][2 + e]);
            }
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        // a row with no key yet keeps its state (every row has key 0 in tile 0)
        const float c0 = mn0 == REF_NEG_INF ? 1.f : expf(m0 - mn0);
        const float c1 = mn1 == REF_NEG_INF ? 1.f : expf(m1 - mn1);
        float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
        for (int n = 0; n < 4; n++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float p0v = sacc[n][e] == REF_NEG_INF ? 0.f : expf(sacc[n][e] - mn0);
                const float p1v = sacc[n][2 + e] == REF_NEG_INF ? 0.f : expf(sacc[n][2 + e] - mn1);
                sacc[n][e] = p0v;
                sacc[n][2 + e] = p1v;
                ps0 += p0v;
                ps1 += p1v;
            }
        }
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
        ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
        ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
        l0 = l0 * c0 + ps0;
        l1 = l1 * c1 + ps1;
        m0 = mn0;
        m1 = mn1;
#pragma unroll
        for (int n = 0; n < 16; n++) {
            o[n][0] *= c0;
            o[n][1] *= c0;
            o[n][2] *= c1;
            o[n][3] *= c1;
        }
        // ---- O += P V: keys in 2 steps of 16, hd in 16 tiles of 8
#pragma unroll
        for (int k2 = 0; k2 < 2; k2++) {
            uint32_t ph[4], pl[4];
            split_h2(sacc[2 * k2][0], sacc[2 * k2][1], ph[0], pl[0]);
            split_h2(sacc[2 * k2][2], sacc[2 * k2][3], ph[1], pl[1]);
            split_h2(sacc[2 * k2 + 1][0], sacc[2 * k2 + 1][1], ph[2], pl[2]);
            split_h2(sacc[2 * k2 + 1][2], sacc[2 * k2 + 1][3], ph[3], pl[3]);
            // keys k2*16 + (t%8) + 8*((t/8)%2), hd nd*16 + 8*(t/16), transposed:
            // (hd tile 2nd: b0, b1), (hd tile 2nd+1: b0, b1)
            const int vrow = k2 * 16 + lrow;
#pragma unroll
            for (int nd = 0; nd < 8; nd++) {
                uint32_t vhf[4], vlf[4];
                ldsm_x4_t(vhf, Vh + vrow * PTC_P + nd * 16 + lcol);
                ldsm_x4_t(vlf, Vl + vrow * PTC_P + nd * 16 + lcol);
                mma_f16(o[2 * nd], ph, vhf[0], vhf[1]);
                mma_f16(o[2 * nd], ph, vlf[0], vlf[1]);
                mma_f16(o[2 * nd], pl, vhf[0], vhf[1]);
                mma_f16(o[2 * nd + 1], ph, vhf[2], vhf[3]);
                mma_f16(o[2 * nd + 1], ph, vlf[2], vlf[3]);
                mma_f16(o[2 * nd + 1], pl, vhf[2], vhf[3]);
            }
        }
        __syncthreads();  // every warp is done with buffer t % 2 before it is refilled
    }
    // ---- normalise and store as the O projection's f16 pair
    const float i0 = 1.0f / l0, i1 = 1.0f / l1;
    const int ra = rw + g, rb = rw + g + 8;
#pragma unroll
    for (int n = 0; n < 16; n++) {
        const int d = 8 * n + 2 * c;
        if (ra < nrows) {
            const size_t oa = (size_t)(r0 + ra) * nh * PTC_HD + (size_t)h * PTC_HD + d;
            split_f16(o[n][0] * i0, xh + oa, xl + oa);
            split_f16(o[n][1] * i0, xh + oa + 1, xl + oa + 1);
        }
        if (rb < nrows) {
            const size_t ob = (size_t)(r0 + rb) * nh * PTC_HD + (size_t)h * PTC_HD + d;
            split_f16(o[n][2] * i1, xh + ob, xl + ob);
            split_f16(o[n][3] * i1, xh + ob + 1, xl + ob + 1);
        }
    }
}

// act = silu(gate) * up or gelu(gate) * up (glu.wgsl:15-32) over the
// interleaved gate/up GEMM output (column 2i gate_i, 2i+1 up_i).
__global__ void k_pf_glu(const float* __restrict__ Gm, int I, int geglu, long rows,
                         __half* __restrict__ xh, __half* __restrict__ xl) {
    pdl_trigger();
    pdl_wait();
    const long n = rows * (long)I;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const long r = i / I, c = i - r * I;
        const float2 gu = *reinterpret_cast<const float2*>(Gm + r * 2 * I + 2 * c);
        const float act = geglu ? gelu_ref_f(gu.x) : silu_ref_f(gu.x);
        split_f16(act * gu.y, xh + i, xl + i);
    }
}

// Hook taps of C prompt rows: row r (stride ld) into ring slot (p0 + r) % cap.
__global__ void k_tap_rows(const float* __restrict__ src, int ld, int len, int rows,
                           float* __restrict__ ring, int cap, int p0) {
    const long n = (long)rows * len;
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n;
         i += (long)gridDim.x * blockDim.x) {
        const int r = (int)(i / len), c = (int)(i - (long)r * len);
        ring[(size_t)((p0 + r) % cap) * len + c] = src[(size_t)r * ld + c];
    }
}

// After the chunk: the next step reads prompt[p_next] at p_next.
__global__ void k_pf_done(DevState* st, const unsigned* __restrict__ prompt, int p_next) {
    st->pos = p_next;
    st->token = prompt[p_next];
}

// ===========================================================================
// host
// ===========================================================================
namespace {

constexpr size_t GEMM_WS_BYTES = 64ull << 20;  // split-K partial tiles of the small-M GEMMs

struct PfLayout {
    size_t H, T, QKV, G, xh, xl, wh, wl, ws, kvp, total;
};

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

// Pair scratch of the tensor-core attention for keys up to max_keys: 4 planes
// [nkv][stride][128] halves, stride = max_keys rounded up to a key tile.
size_t pf_kv_pairs_bytes(int nkv, int max_keys) {
    const size_t stride = (size_t)(max_keys + PTC_BK - 1) / PTC_BK * PTC_BK;
    return 4 * (size_t)nkv * stride * PTC_HD * sizeof(__half);
}

PfLayout pf_layout(const cw_model* m, size_t C, size_t max_keys) {
    const cw_model_info& I = m->info;
    const size_t qd = (size_t)I.n_heads * I.head_dim, kvd = (size_t)I.n_kv * I.head_dim;
    const size_t qkv = qd + 2 * kvd;
    const size_t xk = std::max({(size_t)I.dim, qd, (size_t)I.hidden});
    PfLayout L{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o += al256(bytes);
        return at;
    };
    // the split-K workspace first: its self-resetting counters must sit at
    // the same address for every chunk size
    L.ws = take(GEMM_WS_BYTES);
    L.H = take(C * I.dim * 4);
    L.T = take(I.post_norms ? C * I.dim * 4 : 0);
    L.QKV = take(C * qkv * 4);
    L.G = take(C * 2 * (size_t)I.hidden * 4);
    L.xh = take(C * xk * 2);
    L.xl = take(C * xk * 2);
    const size_t wmax = std::max({qkv * I.dim, (size_t)I.dim * qd, 2 * (size_t)I.hidden * I.dim,
                                  (size_t)I.dim * I.hidden});
    L.wh = take(C > 256 ? wmax * 2 : 0);  // f16 pair of one weight (long chunks)
    L.wl = take(C > 256 ? wmax * 2 : 0);
    // the tensor-core attention's key/value pairs (head_dim 128 families)
    L.kvp = take(I.head_dim == 128 ? pf_kv_pairs_bytes((int)I.n_kv, (int)max_keys) : 0);
    L.total = o;
    return L;
}

template <int EPL, int GM>
int pf_attn_go(cw_ctx* ctx, dim3 grid, size_t smem, const float* QKV, int ld, const float* kc,
               const float* vc, int max_seq, int p0, int nh, int nkv, int hd, int window,
               float scale, float softcap, void* xh, void* xl) {
    if (smem > 48 * 1024)
        CW_CUDA(cudaFuncSetAttribute(k_pf_attn<EPL, GM>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k_pf_attn<EPL, GM><<<grid, 128, smem, ctx->stream>>>(QKV, ld, kc, vc, max_seq, p0, nh, nkv, hd,
                                                          window, scale, softcap, (__half*)xh,
                                                          (__half*)xl);
    return check_launch("prefill attention");
}

template <int EPL>
int pf_attn_e(cw_ctx* ctx, int G, dim3 grid, size_t smem, const float* QKV, int ld,
              const float* kc, const float* vc, int max_seq, int p0, int nh, int nkv, int hd,
              int window, float scale, float softcap, void* xh, void* xl) {
#define CW_PFA(GM)                                                                              \
    return pf_attn_go<EPL, GM>(ctx, grid, smem, QKV, ld, kc, vc, max_seq, p0, nh, nkv, hd, window, \
                               scale, softcap, xh, xl)
    if (G <= 1) CW_PFA(1);
    if (G <= 2) CW_PFA(2);
    if (G <= 4) CW_PFA(4);
    CW_PFA(8);
#undef CW_PFA
}

template <int HD>
int pf_fattn_go(cw_ctx* ctx, int C, const float* QKV, int ld, const float* kc, const float* vc,
                int max_seq, int p0, int nh, int nkv, int window, float scale, float softcap,
                void* xh, void* xl) {
    const size_t smem = pfa_smem(HD);
    if (smem > 48 * 1024)
        CW_CUDA(cudaFuncSetAttribute(k_pf_fattn<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    dim3 grid((C + PFA_BQ - 1) / PFA_BQ, nh);
    k_pf_fattn<HD><<<grid, 256, smem, ctx->stream>>>(QKV, ld, kc, vc, max_seq, p0, C, nh, nkv,
                                                     window, scale, softcap, (__half*)xh,
                                                     (__half*)xl);
    return check_launch("prefill tiled attention");
}

// The tensor-core kernel's layers: head_dim 128, no window, no soft-cap.
bool pf_attn_tc_ok(int hd, int window, float softcap) {
    return hd == PTC_HD && window <= 0 && !(softcap > 0.f);
}

int pf_fattn(cw_ctx* ctx, int hd, int C, const float* QKV, int ld, const float* kc,
             const float* vc, int max_seq, int p0, int nh, int nkv, int window, float scale,
             float softcap, void* xh, void* xl, void* kvp) {
    if (kvp && pf_attn_tc_ok(hd, window, softcap)) {  // the tensor-core kernel
        static thread_local int attr_dev = -1;
        if (attr_dev != ctx->device) {
            CW_CUDA(cudaFuncSetAttribute(k_pf_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)PTC_SMEM));
            attr_dev = ctx->device;
        }
        const int stride = (max_seq + PTC_BK - 1) / PTC_BK * PTC_BK;
        const int n = p0 + C, n_pad = (n + PTC_BK - 1) / PTC_BK * PTC_BK;
        const long items = (long)nkv * n_pad * (PTC_HD / 4);
        const int blocks = (int)std::min<long>((items + 255) / 256, (long)ctx->sm_count * 8);
        k_pf_kv_pairs<<<blocks, 256, 0, ctx->stream>>>(kc, vc, max_seq, nkv, n, n_pad, stride,
                                                        (__half*)kvp);
        CW_TRY(check_launch("prefill key/value pairs"));
        dim3 grid((C + PTC_BQ - 1) / PTC_BQ, nh);
        k_pf_attn_tc<<<grid, 128, PTC_SMEM, ctx->stream>>>(QKV, ld, (const __half*)kvp, stride, p0,
                                                           C, nh, nkv, scale, (__half*)xh,
                                                           (__half*)xl);
        return check_launch("prefill attention (tensor cores)");
    }
    if (hd == 64)
        return pf_fattn_go<64>(ctx, C, QKV, ld, kc, vc, max_seq, p0, nh, nkv, window, scale,
                               softcap, xh, xl);
    if (hd == 128)
        return pf_fattn_go<128>(ctx, C, QKV, ld, kc, vc, max_seq, p0, nh, nkv, window, scale,
                                softcap, xh, xl);
    return pf_fattn_go<256>(ctx, C, QKV, ld, kc, vc, max_seq, p0, nh, nkv, window, scale, softcap,
                            xh, xl);
}

int pf_chunk(cw_session* s, int p0, int C) {
    cw_model* m = s->m;
    cw_ctx* ctx = s->ctx;
    const cw_model_info& I = m->info;
    const int dim = (int)I.dim, nh = (int)I.n_heads, nkv = (int)I.n_kv, hd = (int)I.head_dim;
    const int qd = nh * hd, kvd = nkv * hd, qkv_rows = qd + 2 * kvd, hid = (int)I.hidden;
    const bool post = I.post_norms != 0;
    const int unit = I.norm_kind == 1;
    const PfLayout L = pf_layout(m, (size_t)C, s->max_seq);
    uint8_t* b = (uint8_t*)s->pf_mem;
    float* H = (float*)(b + L.H);
    float* T = (float*)(b + L.T);
    float* QKV = (float*)(b + L.QKV);
    float* Gm = (float*)(b + L.G);
    void *xh = b + L.xh, *xl = b + L.xl, *wh = b + L.wh, *wl = b + L.wl;

    std::unique_ptr<OpScope> sc;
    auto stage = [&](const char* name) {
        sc.reset();
        if (ctx->profiling) sc.reset(new OpScope(ctx, name));
    };
    // Long chunks: each weight is split into its f16 pair once per chunk and the
    // GEMM streams the pair (fastest at large M: the MMA pipe is the bound and
    // shared memory carries only TMA traffic).  Short chunks (<= 256 rows):
    // the weights' packed Q4_0 records, dequantised in shared memory.
    const bool short_chunk = C <= 256;
    if (short_chunk) CW_TRY(model_pack_weights(m));
    int widx = 0;  // layer-major index into m->packed
    auto gemm = [&](const QW& w, int K, int N, float* y, const float* bias, int epi) {
        float* ws = (float*)(b + L.ws);
        if (short_chunk) {
            stage("prefill.gemm");
            return gemm_q4(ctx, xh, xl, m->packed[widx++], C, N, K, y, N, bias, epi, ws,
                           GEMM_WS_BYTES);
        }
        widx++;
        stage("prefill.split_w");
        CW_TRY(q4_split(ctx, w.payload, w.scales, N, K, wh, wl));
        stage("prefill.gemm");
        return gemm_x3(ctx, xh, xl, wh, wl, C, N, K, y, N, bias, epi);
    };
    const int ew_grid = std::max(1, std::min(C * 8, ctx->sm_count * 8));
    auto tap = [&](int kind, uint32_t li, const float* src, int ld) {
        const Tap* t = find_tap(s, kind, li);
        if (!t) return (int)CW_OK;
        k_tap_rows<<<ew_grid, 256, 0, ctx->stream>>>(src, ld, (int)t->len, C, t->ring, (int)t->cap,
                                                     p0);
        return check_launch("prefill hook tap");
    };
    const uint32_t last = I.n_layers - 1;
    const bool last_full = find_tap(s, TAP_POST_ATTN, last) || find_tap(s, TAP_LAYER_OUT, last);

    stage("prefill.embed");
    k_pf_embed<<<C, 256, 0, ctx->stream>>>(m->embed.payload, m->embed.scales, m->embed.type,
                                           dim, I.embed_scale, s->prompt + p0, H);
    CW_TRY(check_launch("prefill embed"));
    for (uint32_t li = 0; li < I.n_layers; li++) {
        const Layer& l = m->L[li];
        widx = 4 * (int)li;  // qkv, wo, gate_up, down
        float* kc = s->kc + (size_t)li * nkv * s->max_seq * hd;
        float* vc = s->vc + (size_t)li * nkv * s->max_seq * hd;
        const bool pre_t = post && li > 0;  // previous layer's FFN output, post-normed in
        stage("prefill.norm");
        k_pf_norm<<<C, 256, dim * 4, ctx->stream>>>(H, pre_t ? T : nullptr,
                                                    pre_t ? m->L[li - 1].post_ffw : nullptr,
                                                    l.attn_norm, unit, I.eps, dim, (__half*)xh,
                                                    (__half*)xl);
        CW_TRY(check_launch("prefill norm"));
        if (pre_t) CW_TRY(tap(TAP_LAYER_OUT, li - 1, H, dim));  // H now holds layer li-1's output
        CW_TRY(gemm(l.qkv, dim, qkv_rows, QKV, l.qkv_bias, GE_STORE));
        stage("prefill.qk");
        k_pf_qk<<<C, 256, 8 * hd * 4, ctx->stream>>>(QKV, qkv_rows, l.q_norm, l.k_norm, I.eps,
                                                      m->inv_freq, kc, vc, (int)s->max_seq, p0,
                                                      nh, nkv, hd);
        CW_TRY(check_launch("prefill qk"));
        CW_TRY(tap(TAP_Q, li, QKV, qkv_rows));
        // only the K/V rows of the last layer are read later (unless tapped)
        if (li == last && !last_full) break;

        stage("prefill.attn");
        const int window = (I.sliding_window && li % 2 == 0) ? (int)I.sliding_window : 0;
        const float scale = powf((float)hd, -0.5f);  // attention.rs:18
        if (hd == 64 || hd == 128 || hd == 256) {
            CW_TRY(pf_fattn(ctx, hd, C, QKV, qkv_rows, kc, vc, (int)s->max_seq, p0, nh, nkv,
                            window, scale, I.attn_softcap, xh, xl, L.kvp ? b + L.kvp : nullptr));
        } else {  // other head sizes: one CTA per (row, kv head)
            const int G = nh / nkv, epl = (hd + 31) / 32;
            const size_t smem = (attn_smem_floats(G, hd, 1) + (size_t)G * hd) * sizeof(float);
            dim3 grid(C, nkv);
#define CW_PFE(E)                                                                              \
    CW_TRY(pf_attn_e<E>(ctx, G, grid, smem, QKV, qkv_rows, kc, vc, (int)s->max_seq, p0, nh, nkv, \
                        hd, window, scale, I.attn_softcap, xh, xl))
            if (epl <= 1) CW_PFE(1);
            else if (epl <= 2) CW_PFE(2);
            else if (epl <= 4) CW_PFE(4);
            else CW_PFE(8);
#undef CW_PFE
        }
        CW_TRY(gemm(l.wo, qd, dim, post ? T : H, nullptr, post ? GE_STORE : GE_ADD));
        if (!post) CW_TRY(tap(TAP_POST_ATTN, li, H, dim));

        stage("prefill.norm");
        k_pf_norm<<<C, 256, dim * 4, ctx->stream>>>(H, post ? T : nullptr,
                                                    post ? l.post_attn : nullptr, l.ffn_norm, unit,
                                                    I.eps, dim, (__half*)xh, (__half*)xl);
        CW_TRY(check_launch("prefill norm"));
        if (post) CW_TRY(tap(TAP_POST_ATTN, li, H, dim));
        CW_TRY(gemm(l.gate_up, dim, 2 * hid, Gm, nullptr, GE_STORE));
        stage("prefill.glu");
        k_pf_glu<<<ew_grid, 256, 0, ctx->stream>>>(Gm, hid, I.activation == 1, C, (__half*)xh,
                                                    (__half*)xl);
        CW_TRY(check_launch("prefill glu"));
        CW_TRY(gemm(l.down, hid, dim, post ? T : H, nullptr, post ? GE_STORE : GE_ADD));
        if (!post) {
            CW_TRY(tap(TAP_LAYER_OUT, li, H, dim));
        } else if (li == last && find_tap(s, TAP_LAYER_OUT, li)) {
            // no next layer folds the post-normed FFN output in: do it for the tap
            k_pf_norm<<<C, 256, dim * 4, ctx->stream>>>(H, T, l.post_ffw, l.ffn_norm, unit, I.eps,
                                                        dim, nullptr, nullptr);
            CW_TRY(check_launch("prefill norm"));
            CW_TRY(tap(TAP_LAYER_OUT, li, H, dim));
        }
    }
    stage("prefill.done");
    k_pf_done<<<1, 1, 0, ctx->stream>>>(s->st, s->prompt, p0 + C);
    sc.reset();
    return check_launch("prefill done");
}

}  // namespace

int session_prefill(cw_session* s, size_t* n_done) {
    const size_t end = s->n_prompt - 1;  // the last prompt token runs through the decode step
    size_t done = 0;
    if (s->host_pos < end) {
        const size_t chunk = s->pf_chunk ? std::min<size_t>(s->pf_chunk, PF_CHUNK) : PF_CHUNK;
        const size_t C = std::min<size_t>(end - s->host_pos, chunk);
        const PfLayout L = pf_layout(s->m, C, s->max_seq);
        if (s->pf_bytes < L.total) {
            CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
            if (s->pf_mem) cudaFree(s->pf_mem);
            s->pf_mem = nullptr;
            s->pf_bytes = 0;
            CW_CUDA(cudaMalloc(&s->pf_mem, L.total));
            CW_CUDA(cudaMemsetAsync(s->pf_mem, 0, L.total, s->ctx->stream));  // split-K counters
            s->pf_bytes = L.total;
        }
        while (s->host_pos < end) {
            const int c = (int)std::min<size_t>(end - s->host_pos, C);
            CW_TRY(pf_chunk(s, (int)s->host_pos, c));
            s->host_pos += c;
            done += c;
        }
    }
    if (n_done) *n_done = done;
    return CW_OK;
}

}  // namespace cw

// ===========================================================================
// co-batched decode: one step of B independent sessions together
// ===========================================================================
// Each row is one session at its own position with its own KV cache; the
// projections of all rows share one pass over the weights as tensor-core
// GEMMs (the f16 pairs of model->split), so the weight stream is paid once
// per step instead of once per session.  Per session the step does exactly
// what its single-session step does (embed, layers, final norm, LM head,
// argmax / sampling / EOS, generate-loop bookkeeping, mod.rs:57-125).
namespace cw {
namespace {

// A plain (uncached) read of a word another kernel may be writing.
__device__ __forceinline__ int ld_volatile_global(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

struct GrpRow {
    DevState* st;
    const unsigned* prompt;
    unsigned* toks;
    float* logits;  // the session's logits buffer (cw_session_logits)
    const SampleParams* smp;
    float *kc, *vc;  // layer-0 cache bases
    int max_seq, pad;
};

__global__ void k_grp_embed(const uint8_t* __restrict__ payload, const __half* __restrict__ scales,
                            int type, int dim, float scale, const GrpRow* __restrict__ rows,
                            float* __restrict__ H) {
    pdl_trigger();
    pdl_wait();
    const int r = blockIdx.x;
    const unsigned tok = rows[r].st->token;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = embed_elem(payload, scales, type, tok, dim, i);
        H[(size_t)r * dim + i] = scale > 0.f ? __fmul_rn(v, scale) : v;
    }
}

// One group step's attention with QK-norm, RoPE and the K/V row write fused
// in front (the single-session k_fattn of cw_model.cu over rows of different
// sessions): CTA (split, kv head g, row r) takes key range `split` of row
// r's live span; the CTA whose range holds the row's position writes its
// K/V row, so no other CTA reads it.  With several splits the last CTA of a
// (row, kv head) merges the partial states (fixed order) and writes the
// output as the f16 hi/lo pair of the O projection.
template <int EPL, int GMAX>
__global__ void __launch_bounds__(128) k_grp_fattn(
    const float* __restrict__ QKV, int ld, const GrpRow* __restrict__ rows, int li,
    const float* __restrict__ q_norm, const float* __restrict__ k_norm, float eps,
    const float* __restrict__ inv_freq, int nh, int nkv, int hd, int n_splits, int window,
    float scale, float softcap, float* __restrict__ part, unsigned* __restrict__ counters,
    __half* __restrict__ xh, __half* __restrict__ xl, float* __restrict__ xo) {
    pdl_trigger();
    extern __shared__ float sm[];
    const int split = blockIdx.x, g = blockIdx.y, r = blockIdx.z;
    const int G = nh / nkv, W = hd + 2, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const GrpRow R = rows[r];  // the row table does not change while a group steps
    const size_t lstride = (size_t)nkv * R.max_seq * hd;
    float* kbase = R.kc + li * lstride + (size_t)g * R.max_seq * hd;
    float* vbase = R.vc + li * lstride + (size_t)g * R.max_seq * hd;
    if (threadIdx.x == 0) {
        // while the QKV projection runs: pull this split's cached K/V rows
        // into L2.  The position may still be the previous step's (a hint
        // only; the range stays inside the cache), the real one is read
        // after the wait.
        const int hpos = min(max(ld_volatile_global(&R.st->pos), 0), R.max_seq - 1), hseq = hpos + 1;
        const int hact = attn_active_splits(attn_span(hseq, window), n_splits);
        if (split < hact) {
            int a0, a1;
            attn_range(hseq, window, split, hact, &a0, &a1);
            a1 = min(a1, hpos);
            if (a1 > a0) {
                prefetch_l2(kbase + (size_t)a0 * hd, kbase + (size_t)a1 * hd);
                prefetch_l2(vbase + (size_t)a0 * hd, vbase + (size_t)a1 * hd);
            }
        }
    }
    pdl_wait();
    const int pos = R.st->pos, seq = pos + 1;
    const int n_active = attn_active_splits(attn_span(seq, window), n_splits);
    if (split >= n_active) return;
    int jlo, jhi;
    attn_range(seq, window, split, n_active, &jlo, &jhi);
    const bool holds = pos >= jlo && pos < jhi;
    float* qs = sm + attn_smem_floats(G, hd, n_splits);  // [G][hd]
    float* ks = qs + (size_t)G * hd;                     // [hd]
    const float* row = QKV + (size_t)r * ld;
    const int qd = nh * hd, kvd = nkv * hd;
    const int nrows = G + (holds ? 1 : 0);
    for (int t = warp; t < nrows; t += 4) {  // QK-norm (qwen3.rs:154-155), one warp per row
        const bool isq = t < G;
        const float* src = isq ? row + (size_t)(g * G + t) * hd : row + qd + (size_t)g * hd;
        const float* nw = isq ? q_norm : k_norm;
        float* dst = isq ? qs + (size_t)t * hd : ks;
        float v[EPL];
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            const int d = lane + 32 * e;
            v[e] = d < hd ? src[d] : 0.f;
            ss = fmaf(v[e], v[e], ss);
        }
        if (nw) {
            ss = warp_sum(ss);
            const float inv = 1.0f / sqrtf(ss / (float)hd + eps);
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                const int d = lane + 32 * e;
                if (d < hd) v[e] = __fmul_rn(__fmul_rn(v[e], inv), nw[d]);
            }
        }
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            const int d = lane + 32 * e;
            if (d < hd) dst[d] = v[e];
        }
    }
    __syncthreads();
    const int half = hd / 2;  // RoPE (rope.wgsl:25-34) in place
    for (int i = threadIdx.x; i < nrows * half; i += blockDim.x) {
        const int t = i / half, k = i - t * half;
        float* rw = t < G ? qs + (size_t)t * hd : ks;
        const float freq = __fmul_rn((float)pos, inv_freq[k]);
        float sn, cs;
        sincosf(freq, &sn, &cs);
        const float lo = rw[k], hi = rw[k + half];
        rw[k] = __fsub_rn(__fmul_rn(lo, cs), __fmul_rn(hi, sn));
        rw[k + half] = __fadd_rn(__fmul_rn(hi, cs), __fmul_rn(lo, sn));
    }
    __syncthreads();
    if (holds) {  // cache.rs:21-24: this position's K (normed, roped) and V
        const float* vsrc = row + qd + kvd + (size_t)g * hd;
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            kbase[(size_t)pos * hd + d] = ks[d];
            vbase[(size_t)pos * hd + d] = vsrc[d];
        }
    }
    __syncthreads();
    float* res = sm + 4 * G * W;
    attn_core<EPL, GMAX, KV_PLAIN>(qs, G, hd, kbase, vbase, hd, jlo, jhi, scale, softcap, sm, res);
    const size_t o0 = (size_t)r * qd + (size_t)g * G * hd;
    if (n_active == 1) {
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
            const int gi = i / hd, d = i - gi * hd;
            const float o = res[gi * W + d] * (1.0f / res[gi * W + hd + 1]);
            if (xo)
                xo[o0 + i] = o;
            else
                split_f16(o, xh + o0 + i, xl + o0 + i);
        }
        return;
    }
    float* pr = part + ((size_t)r * nh + (size_t)g * G) * n_splits * W;  // [G][n_splits][W]
    for (int i = threadIdx.x; i < G * W; i += blockDim.x) {
        const int gi = i / W, d = i - gi * W;
        pr[((size_t)gi * n_splits + split) * W + d] = res[i];
    }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    unsigned* ctr = counters + (size_t)r * nkv + g;
    if (threadIdx.x == 0) s_last = atomicAdd(ctr, 1u) == (unsigned)n_active - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    float* cwt = sm;  // merge weights [G][n_active + 1]
    for (int gi = warp; gi < G; gi += 4) {
        const float* ph = pr + (size_t)gi * n_splits * W;
        float M = REF_NEG_INF;
        for (int t = lane; t < n_active; t += 32) M = fmaxf(M, __ldcg(ph + (size_t)t * W + hd));
        M = warp_max(M);
        float L = 0.f;
        for (int t = lane; t < n_active; t += 32) {
            const float c = expf(__ldcg(ph + (size_t)t * W + hd) - M);
            cwt[gi * (n_active + 1) + t] = c;
            L += __ldcg(ph + (size_t)t * W + hd + 1) * c;
        }
        L = warp_sum(L);
        if (lane == 0) cwt[gi * (n_active + 1) + n_active] = 1.0f / L;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        const int gi = i / hd, d = i - gi * hd;
        const float* ph = pr + (size_t)gi * n_splits * W + d;
        const float* c = cwt + gi * (n_active + 1);
        float a = 0.f;
        for (int t = 0; t < n_active; t++) a = fmaf(__ldcg(ph + (size_t)t * W), c[t], a);
        if (xo)
            xo[o0 + i] = a * c[n_active];
        else
            split_f16(a * c[n_active], xh + o0 + i, xl + o0 + i);
    }
    __syncthreads();
    if (threadIdx.x == 0) *ctr = 0u;
}

// Per session: soft-capped logits into its buffer, argmax (ties -> lowest,
// argmax.wgsl), then the generate-loop bookkeeping of its own step
// (mod.rs:114-122) with sampling and stop tokens as cw_sample.cu applies them.
__global__ void __launch_bounds__(SMP_THREADS) k_grp_finalize(const GrpRow* __restrict__ rows,
                                                              const float* __restrict__ logits,
                                                              int V, float softcap) {
    pdl_trigger();
    pdl_wait();
    __shared__ SmpShared S;
    __shared__ unsigned long long best[SMP_THREADS / 32];
    const GrpRow R = rows[blockIdx.x];
    const float* lr = logits + (size_t)blockIdx.x * V;
    unsigned long long k = argmax_key_init();
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        float v = lr[i];
        if (softcap > 0.f) v = softcap * tanhf(v / softcap);
        R.logits[i] = v;
        const unsigned long long c = argmax_key(v, (unsigned)i);
        k = c > k ? c : k;
    }
    for (int o = 16; o; o >>= 1) {
        const unsigned long long c = __shfl_xor_sync(0xffffffffu, k, o);
        k = c > k ? c : k;
    }
    if ((threadIdx.x & 31) == 0) best[threadIdx.x >> 5] = k;
    __syncthreads();
    k = best[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) k = best[w] > k ? best[w] : k;
    const unsigned amax = argmax_key_index(k);
    DevState* st = R.st;
    const int pos = st->pos;
    __syncthreads();
    if (pos + 1 < st->n_prompt) {  // a prompt position: the next input is the next prompt token
        if (threadIdx.x == 0) {
            st->token = R.prompt[pos + 1];
            st->pos = pos + 1;
        }
        return;
    }
    const SampleParams p = *R.smp;
    const int np = st->n_produced;
    const unsigned t = sample_core(S, R.logits, V, p, (unsigned long long)np, amax);
    if (threadIdx.x == 0) {
        if (!st->stopped) {
            bool eos = false;
            for (unsigned j = 0; j < p.n_eos; j++) eos |= p.eos[j] == t;
            if (eos) {
                st->stopped = 1;
            } else {
                R.toks[np] = t;
                st->n_produced = np + 1;
            }
        }
        st->token = t;
        st->pos = pos + 1;
    }
}

// The streaming path's finalize: the head GEMV already stored each session's
// soft-capped logits and reduced its argmax key into keys[r]; here the
// generate-loop bookkeeping of each session (mod.rs:114-122) with sampling
// and stop tokens as cw_sample.cu applies them, and the key reset for the
// next step.
__global__ void __launch_bounds__(SMP_THREADS) k_grp_finalize_keys(const GrpRow* __restrict__ rows,
                                                                   unsigned long long* keys, int V) {
    pdl_trigger();
    pdl_wait();
    __shared__ SmpShared S;
    const GrpRow R = rows[blockIdx.x];
    const unsigned amax = argmax_key_index(keys[blockIdx.x]);
    DevState* st = R.st;
    const int pos = st->pos;
    __syncthreads();
    if (threadIdx.x == 0) keys[blockIdx.x] = argmax_key_init();
    if (pos + 1 < st->n_prompt) {  // a prompt position: the next input is the next prompt token
        if (threadIdx.x == 0) {
            st->token = R.prompt[pos + 1];
            st->pos = pos + 1;
        }
        return;
    }
    const SampleParams p = *R.smp;
    const int np = st->n_produced;
    const unsigned t = sample_core(S, R.logits, V, p, (unsigned long long)np, amax);
    if (threadIdx.x == 0) {
        if (!st->stopped) {
            bool eos = false;
            for (unsigned j = 0; j < p.n_eos; j++) eos |= p.eos[j] == t;
            if (eos) {
                st->stopped = 1;
            } else {
                R.toks[np] = t;
                st->n_produced = np + 1;
            }
        }
        st->token = t;
        st->pos = pos + 1;
    }
}

struct GrpLayout {
    size_t H, T, QKV, G, xh, xl, X, logits, ws, part, ctr, yrow, keys, total;
};

// Key splits of the group attention: about four CTAs per SM over all rows and
// kv heads (at most 16).
int grp_splits(const cw_model* m, size_t B, int sm_count) {
    const int per = (int)(4 * sm_count / std::max<size_t>(1, B * m->info.n_kv));
    return std::max(1, std::min(16, per));
}

GrpLayout grp_layout(const cw_model* m, size_t B) {
    const cw_model_info& I = m->info;
    const size_t qd = (size_t)I.n_heads * I.head_dim, kvd = (size_t)I.n_kv * I.head_dim;
    const size_t xk = std::max({(size_t)I.dim, qd, (size_t)I.hidden});
    GrpLayout L{};
    size_t o = 0;
    auto take = [&](size_t bytes) {
        size_t at = o;
        o += al256(bytes);
        return at;
    };
    L.ws = take(GEMM_WS_BYTES);  // first, as in the prefill layout
    L.H = take(B * I.dim * 4);
    L.T = take(B * I.dim * 4);
    L.QKV = take(B * (qd + 2 * kvd) * 4);
    L.G = take(B * 2 * (size_t)I.hidden * 4);
    L.xh = take(B * xk * 2);
    L.xl = take(B * xk * 2);
    L.X = take(B * qd * 4);
    L.logits = take(B * (size_t)I.vocab * 4);
    L.part = take(B * (size_t)I.n_heads * 16 * (I.head_dim + 2) * 4);  // up to 16 splits
    L.ctr = take(B * (size_t)I.n_kv * 4);  // merge counters (zero, self-resetting)
    L.yrow = take(B * sizeof(float*));     // each session's logits buffer (streaming head)
    L.keys = take(B * 8);                  // each session's argmax key (streaming head)
    L.total = o;
    return L;
}

}  // namespace

int model_pack_weights(cw_model* m) {
    if (!m->packed.empty()) return CW_OK;
    cw_ctx* ctx = m->ctx;
    std::vector<void*> out;
    auto add = [&](const QW& w) -> int {
        void* p = nullptr;
        CW_CUDA(cudaMalloc(&p, q4_tile_bytes(w.rows, w.in_f)));
        out.push_back(p);
        return q4_tile_pack(ctx, w.payload, w.scales, w.rows, w.in_f, p);
    };
    int rc = CW_OK;
    for (const Layer& l : m->L) {
        for (const QW* w : {&l.qkv, &l.wo, &l.gate_up, &l.down})
            if (rc == CW_OK) rc = add(*w);
    }
    if (rc == CW_OK && m->head.type == 2) rc = add(m->head);  // a Q6_K head has no record form
    if (rc == CW_OK && cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        rc = set_error(CW_ERR_CUDA, "weight packing failed");
    if (rc != CW_OK) {
        for (void* p : out) cudaFree(p);
        return rc;
    }
    m->packed = out;
    return CW_OK;
}

}  // namespace cw

struct cw_group {
    cw_model* m = nullptr;
    int n_splits = 1;  // key splits of the attention
    std::vector<cw_session*> ss;
    cw::GrpRow* rows = nullptr;  // device
    void* mem = nullptr;         // scratch (GrpLayout)
    cudaGraphExec_t graph = nullptr;
    // projections as co-batched streaming GEMVs (cw_mgemv.cu) instead of
    // tensor-core GEMMs over the packed tile records; their products on the
    // integer MMA where K allows (else dp4a)
    bool streaming = false;
    bool mma = true;
};

namespace cw {

// The co-batched step with every projection a streaming GEMV over all rows
// (cw_mgemv.cu): 5 launches per layer -- norm + QKV, attention, O +
// residual, norm + gate/up + GLU, down + residual -- each one pass over its
// weight for all sessions.
static int grp_enqueue_streaming(cw_group* g) {
    cw_model* m = g->m;
    cw_ctx* ctx = m->ctx;
    const cw_model_info& I = m->info;
    const int B = (int)g->ss.size();
    const int dim = (int)I.dim, nh = (int)I.n_heads, nkv = (int)I.n_kv, hd = (int)I.head_dim;
    const int qd = nh * hd, kvd = nkv * hd, qkv_rows = qd + 2 * kvd, hid = (int)I.hidden;
    const int unit = I.norm_kind == 1;
    const GrpLayout L = grp_layout(m, (size_t)B);
    uint8_t* b = (uint8_t*)g->mem;
    float* H = (float*)(b + L.H);
    float* QKV = (float*)(b + L.QKV);
    float* A = (float*)(b + L.G);  // FFN activations [B][hid]
    float* X = (float*)(b + L.X);  // attention output [B][qd]
    float* logits = (float*)(b + L.logits);
    std::unique_ptr<OpScope> sc;
    auto stage = [&](const char* name) {
        sc.reset();
        if (ctx->profiling) sc.reset(new OpScope(ctx, name));
    };
    auto mg = [&](const char* name, int widx, const QW& w, int pro, int epi, const float* x,
                  int ldx, const float* norm_w, float* y, int ldy, const float* bias) {
        stage(name);
        MgArgs a{};
        a.tiles = (const uint8_t*)m->grp_tiles[widx];
        a.payload = w.payload;
        a.scales = w.scales;
        a.K = w.in_f;
        a.N = w.rows;
        a.B = B;
        a.x = x;
        a.ldx = ldx;
        a.norm_w = norm_w;
        a.eps = I.eps;
        a.unit = unit;
        a.y = y;
        a.ldy = ldy;
        a.bias = bias;
        a.geglu = I.activation == 1;
        a.status = ctx->d_status;
        a.mma = g->mma ? 1 : 0;
        CW_TRY(launch_mgemv(ctx, pro, epi, a, true));
        return check_launch(name);
    };
    stage("group.embed");
    CW_TRY(launch_pdl(ctx, true, k_grp_embed, dim3(B), dim3(256), 0, m->embed.payload,
                      m->embed.scales, m->embed.type, dim, I.embed_scale, (const GrpRow*)g->rows,
                      H));
    CW_TRY(check_launch("group embed"));
    for (uint32_t li = 0; li < I.n_layers; li++) {
        const Layer& l = m->L[li];
        CW_TRY(mg("group.qkv", 4 * li + 0, l.qkv, PRO_NORM, EPI_STORE, H, dim, l.attn_norm, QKV, qkv_rows,
                  l.qkv_bias));
        stage("group.attn");
        {
            const int G = nh / nkv, epl = (hd + 31) / 32, ns = g->n_splits;
            const size_t smem =
                (attn_smem_floats(G, hd, ns) + (size_t)G * hd + hd) * sizeof(float);
            const int window = (I.sliding_window && li % 2 == 0) ? (int)I.sliding_window : 0;
            const float scale = powf((float)hd, -0.5f);  // attention.rs:18
            dim3 grid(ns, nkv, B);
            float* part = (float*)(b + L.part);
            unsigned* ctr = (unsigned*)(b + L.ctr);
            auto go = [&](auto kern) -> int {
                if (smem > 48 * 1024)
                    CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem));
                CW_TRY(launch_pdl(ctx, true, kern, grid, dim3(128), smem, (const float*)QKV,
                                  qkv_rows, (const GrpRow*)g->rows, (int)li,
                                  (const float*)l.q_norm, (const float*)l.k_norm, I.eps,
                                  m->inv_freq, nh, nkv, hd, ns, window, scale, I.attn_softcap,
                                  part, ctr, (__half*)nullptr, (__half*)nullptr, X));
                return check_launch("group attention");
            };
#define CW_GA(E, GM) CW_TRY(go(k_grp_fattn<E, GM>))
#define CW_GAE(E)                 \
    if (G <= 1) CW_GA(E, 1);      \
    else if (G <= 2) CW_GA(E, 2); \
    else if (G <= 4) CW_GA(E, 4); \
    else CW_GA(E, 8);
            if (epl <= 1) { CW_GAE(1) }
            else if (epl <= 2) { CW_GAE(2) }
            else if (epl <= 4) { CW_GAE(4) }
            else { CW_GAE(8) }
#undef CW_GAE
#undef CW_GA
        }
        CW_TRY(mg("group.o", 4 * li + 1, l.wo, PRO_X, EPI_RESID, X, qd, nullptr, H, dim, nullptr));
        CW_TRY(mg("group.gate_up", 4 * li + 2, l.gate_up, PRO_NORM, EPI_GLU, H, dim, l.ffn_norm, A, hid,
                  nullptr));
        CW_TRY(mg("group.down", 4 * li + 3, l.down, PRO_X, EPI_RESID, A, hid, nullptr, H, dim, nullptr));
    }
    if (dim / 32 <= 128) {
        // the head's epilogue soft-caps, stores each session's logits and
        // reduces its argmax key; finalize only does the bookkeeping (and
        // samples where a session asks for it)
        stage("group.head");
        MgArgs a{};
        a.tiles = (const uint8_t*)m->grp_tiles[4 * I.n_layers];
        a.payload = m->head.payload;
        a.scales = m->head.scales;
        a.K = m->head.in_f;
        a.N = m->head.rows;
        a.B = B;
        a.x = H;
        a.ldx = dim;
        a.norm_w = m->final_norm;
        a.eps = I.eps;
        a.unit = unit;
        a.status = ctx->d_status;
        a.mma = 1;
        a.yrow = (float* const*)(b + L.yrow);
        a.keys = (unsigned long long*)(b + L.keys);
        a.softcap = I.final_softcap;
        CW_TRY(launch_mgemv(ctx, PRO_NORM, EPI_HEAD, a, true));
        CW_TRY(check_launch("group head"));
        stage("group.finalize");
        CW_TRY(launch_pdl(ctx, true, k_grp_finalize_keys, dim3(B), dim3(SMP_THREADS), 0,
                          (const GrpRow*)g->rows, (unsigned long long*)(b + L.keys), (int)I.vocab));
        sc.reset();
        return check_launch("group finalize");
    }
    CW_TRY(mg("group.head", 4 * I.n_layers, m->head, PRO_NORM, EPI_STORE, H, dim, m->final_norm, logits,
              (int)I.vocab, nullptr));
    stage("group.finalize");
    CW_TRY(launch_pdl(ctx, true, k_grp_finalize, dim3(B), dim3(SMP_THREADS), 0,
                      (const GrpRow*)g->rows, (const float*)logits, (int)I.vocab,
                      I.final_softcap));
    sc.reset();
    return check_launch("group finalize");
}

// Whether a group of B sessions can take the streaming step: pre-norm
// families (post-norm residuals would need a second residual buffer), at
// most 8 sessions, every projection's K a multiple of 256 within the
// kernel's range.
static bool grp_streaming_ok(const cw_model* m, size_t B) {
    const cw_model_info& I = m->info;
    const int qd = (int)(I.n_heads * I.head_dim);
    return I.post_norms == 0 && mgemv_supported((int)I.dim, (int)B) &&
           mgemv_supported(qd, (int)B) && mgemv_supported((int)I.hidden, (int)B);
}

// The tile-interleaved weight copies of the streaming step (model->grp_tiles:
// 4 per layer, then the head), idempotent; matrices whose K is beyond the
// integer-MMA path keep a null entry.
static int model_tile_weights(cw_model* m) {
    if (!m->grp_tiles.empty()) return CW_OK;
    cw_ctx* ctx = m->ctx;
    std::vector<void*> out;
    auto add = [&](const QW& w) -> int {
        void* p = nullptr;
        if (w.in_f / 32 <= 128) {
            CW_CUDA(cudaMalloc(&p, mg_tile_bytes(w.rows, w.in_f)));
            out.push_back(p);
            return mg_tile_pack(ctx, w.payload, w.scales, w.rows, w.in_f, p);
        }
        out.push_back(nullptr);
        return CW_OK;
    };
    int rc = CW_OK;
    for (const Layer& l : m->L)
        for (const QW* w : {&l.qkv, &l.wo, &l.gate_up, &l.down})
            if (rc == CW_OK) rc = add(*w);
    if (rc == CW_OK) rc = add(m->head);
    if (rc == CW_OK && cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        rc = set_error(CW_ERR_CUDA, "weight tiling failed");
    if (rc != CW_OK) {
        for (void* p : out) cudaFree(p);
        return rc;
    }
    m->grp_tiles = out;
    return CW_OK;
}

static int grp_enqueue(cw_group* g) {
    if (g->streaming) return grp_enqueue_streaming(g);
    cw_model* m = g->m;
    cw_ctx* ctx = m->ctx;
    const cw_model_info& I = m->info;
    const int B = (int)g->ss.size();
    const int dim = (int)I.dim, nh = (int)I.n_heads, nkv = (int)I.n_kv, hd = (int)I.head_dim;
    const int qd = nh * hd, kvd = nkv * hd, qkv_rows = qd + 2 * kvd, hid = (int)I.hidden;
    const bool post = I.post_norms != 0;
    const int unit = I.norm_kind == 1;
    const GrpLayout L = grp_layout(m, (size_t)B);
    uint8_t* b = (uint8_t*)g->mem;
    float* H = (float*)(b + L.H);
    float* T = (float*)(b + L.T);
    float* QKV = (float*)(b + L.QKV);
    float* Gm = (float*)(b + L.G);
    float* logits = (float*)(b + L.logits);
    void *xh = b + L.xh, *xl = b + L.xl;
    std::unique_ptr<OpScope> sc;
    auto stage = [&](const char* name) {
        sc.reset();
        if (ctx->profiling) sc.reset(new OpScope(ctx, name));
    };
    auto gemm = [&](int widx, int K, int N, float* y, const float* bias, int epi) {
        stage(widx == 4 * (int)I.n_layers ? "group.gemm_head" : "group.gemm");
        return gemm_q4(ctx, xh, xl, m->packed[widx], B, N, K, y, N, bias, epi,
                       (float*)(b + L.ws), GEMM_WS_BYTES, true);
    };
    const int ew_grid = std::max(1, std::min(B * 8, ctx->sm_count * 8));
    stage("group.embed");
    CW_TRY(launch_pdl(ctx, true, k_grp_embed, dim3(B), dim3(256), 0, m->embed.payload,
                      m->embed.scales, m->embed.type, dim, I.embed_scale, (const GrpRow*)g->rows,
                      H));
    CW_TRY(check_launch("group embed"));
    for (uint32_t li = 0; li < I.n_layers; li++) {
        const Layer& l = m->L[li];
        const bool pre_t = post && li > 0;
        stage("group.norm");
        CW_TRY(launch_pdl(ctx, true, k_pf_norm, dim3(B), dim3(256), (size_t)dim * 4, H, pre_t ? T : nullptr,
                                                    pre_t ? m->L[li - 1].post_ffw : nullptr,
                                                    l.attn_norm, unit, I.eps, dim, (__half*)xh,
                                                    (__half*)xl));
        CW_TRY(check_launch("group norm"));
        CW_TRY(gemm(4 * li + 0, dim, qkv_rows, QKV, l.qkv_bias, GE_STORE));
        stage("group.attn");
        {
            const int G = nh / nkv, epl = (hd + 31) / 32, ns = g->n_splits;
            const size_t smem =
                (attn_smem_floats(G, hd, ns) + (size_t)G * hd + hd) * sizeof(float);
            const int window = (I.sliding_window && li % 2 == 0) ? (int)I.sliding_window : 0;
            const float scale = powf((float)hd, -0.5f);  // attention.rs:18
            dim3 grid(ns, nkv, B);
            float* part = (float*)(b + L.part);
            unsigned* ctr = (unsigned*)(b + L.ctr);
            auto go = [&](auto kern) -> int {
                if (smem > 48 * 1024)
                    CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 (int)smem));
                CW_TRY(launch_pdl(ctx, true, kern, grid, dim3(128), smem, (const float*)QKV,
                                  qkv_rows, (const GrpRow*)g->rows, (int)li,
                                  (const float*)l.q_norm, (const float*)l.k_norm, I.eps,
                                  m->inv_freq, nh, nkv, hd, ns, window, scale, I.attn_softcap,
                                  part, ctr, (__half*)xh, (__half*)xl, (float*)nullptr));
                return check_launch("group attention");
            };
#define CW_GA(E, GM) CW_TRY(go(k_grp_fattn<E, GM>))
#define CW_GAE(E)                 \
    if (G <= 1) CW_GA(E, 1);      \
    else if (G <= 2) CW_GA(E, 2); \
    else if (G <= 4) CW_GA(E, 4); \
    else CW_GA(E, 8);
            if (epl <= 1) { CW_GAE(1) }
            else if (epl <= 2) { CW_GAE(2) }
            else if (epl <= 4) { CW_GAE(4) }
            else { CW_GAE(8) }
#undef CW_GAE
#undef CW_GA
        }
        CW_TRY(gemm(4 * li + 1, qd, dim, post ? T : H, nullptr, post ? GE_STORE : GE_ADD));
        stage("group.norm");
        CW_TRY(launch_pdl(ctx, true, k_pf_norm, dim3(B), dim3(256), (size_t)dim * 4, H, post ? T : nullptr,
                                                    post ? l.post_attn : nullptr, l.ffn_norm, unit,
                                                    I.eps, dim, (__half*)xh, (__half*)xl));
        CW_TRY(check_launch("group norm"));
        CW_TRY(gemm(4 * li + 2, dim, 2 * hid, Gm, nullptr, GE_STORE));
        stage("group.glu");
        CW_TRY(launch_pdl(ctx, true, k_pf_glu, dim3(ew_grid), dim3(256), 0, (const float*)Gm, hid,
                          (int)(I.activation == 1), (long)B, (__half*)xh, (__half*)xl));
        CW_TRY(check_launch("group glu"));
        CW_TRY(gemm(4 * li + 3, hid, dim, post ? T : H, nullptr, post ? GE_STORE : GE_ADD));
    }
    // final norm (post-norm families: the last FFN output folded in first), head, finalize
    stage("group.norm");
    CW_TRY(launch_pdl(ctx, true, k_pf_norm, dim3(B), dim3(256), (size_t)dim * 4, H, post ? T : nullptr,
                                                post ? m->L[I.n_layers - 1].post_ffw : nullptr,
                                                m->final_norm, unit, I.eps, dim, (__half*)xh,
                                                (__half*)xl));
    CW_TRY(check_launch("group final norm"));
    CW_TRY(gemm(4 * (int)I.n_layers, dim, (int)I.vocab, logits, nullptr, GE_STORE));
    stage("group.finalize");
    CW_TRY(launch_pdl(ctx, true, k_grp_finalize, dim3(B), dim3(SMP_THREADS), 0,
                      (const GrpRow*)g->rows, (const float*)logits, (int)I.vocab,
                      I.final_softcap));
    sc.reset();
    return check_launch("group finalize");
}

static int grp_step(cw_group* g) {
    for (cw_session* s : g->ss)
        CW_CHECK(s->host_pos < s->max_seq, CW_ERR_INVALID_ARG,
                 "group step: a session is full (position %zu, max_seq %zu)", s->host_pos,
                 s->max_seq);
    cw_ctx* ctx = g->m->ctx;
    if (ctx->profiling) {  // direct launches, each stage bracketed by profiler events
        CW_TRY(grp_enqueue(g));
    } else if (!g->graph) {
        cudaGraph_t gr = nullptr;
        CW_CUDA(cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal));
        int rc = grp_enqueue(g);
        cudaError_t e = cudaStreamEndCapture(ctx->stream, &gr);
        if (rc != CW_OK) {
            if (gr) cudaGraphDestroy(gr);
            return rc;
        }
        if (e != cudaSuccess) return set_error(CW_ERR_CUDA, "group capture: %s", cudaGetErrorString(e));
        e = cudaGraphInstantiate(&g->graph, gr, 0);
        cudaGraphDestroy(gr);
        if (e != cudaSuccess)
            return set_error(CW_ERR_CUDA, "group instantiate: %s", cudaGetErrorString(e));
    }
    if (!ctx->profiling) CW_CUDA(cudaGraphLaunch(g->graph, ctx->stream));
    for (cw_session* s : g->ss) {
        if (s->host_pos + 1 >= s->n_prompt) s->n_produced++;
        s->host_pos++;
    }
    return CW_OK;
}

static int grp_sync(cw_group* g) {
    for (cw_session* s : g->ss) CW_TRY(sync_counts(s));
    return CW_OK;
}

}  // namespace cw

using namespace cw;

extern "C" {

int cw_group_create(cw_session* const* sessions, size_t n, cw_group** out) {
    clear_error();
    CW_CHECK(sessions && out && n > 0 && n <= 1024, CW_ERR_INVALID_ARG,
             "cw_group_create: 1..1024 sessions");
    cw_model* m = sessions[0] ? sessions[0]->m : nullptr;
    CW_CHECK(m, CW_ERR_INVALID_ARG, "cw_group_create: NULL session");
    for (size_t i = 0; i < n; i++) {
        CW_CHECK(sessions[i] && sessions[i]->m == m, CW_ERR_INVALID_ARG,
                 "cw_group_create: sessions must share one model");
        for (size_t j = 0; j < i; j++)
            CW_CHECK(sessions[j] != sessions[i], CW_ERR_INVALID_ARG,
                     "cw_group_create: a session appears twice");
    }
    cw_ctx* ctx = m->ctx;
    CW_CHECK(m->tp_world == 1, CW_ERR_UNSUPPORTED,
             "cw_group_create: not available on a tensor-parallel model");
    CW_CHECK(model_q4_only(m, true), CW_ERR_UNSUPPORTED,
             "cw_group_create: the co-batched step takes Q4_0 projections and LM head");
    cudaSetDevice(ctx->device);
    const bool streaming = grp_streaming_ok(m, n);
    CW_TRY(streaming ? model_tile_weights(m) : model_pack_weights(m));
    cw_group* g = new cw_group();
    g->m = m;
    g->streaming = streaming;
    g->n_splits = grp_splits(m, n, ctx->sm_count);
    g->ss.assign(sessions, sessions + n);
    std::vector<GrpRow> h(n);
    std::vector<float*> yrow(n);
    // argmax_key_init(): the reference's start value -3.402823e38 at index 0
    // (argmax.wgsl:23), as the order-preserving key of cw_device.cuh
    float start = -3.402823e38f;
    uint32_t sbits;
    memcpy(&sbits, &start, 4);
    const uint64_t kinit = ((uint64_t)(~sbits) << 32) | 0xffffffffull;
    std::vector<uint64_t> keys(n, kinit);
    for (size_t i = 0; i < n; i++) {
        cw_session* s = sessions[i];
        h[i] = GrpRow{s->st, s->prompt, s->toks, s->logits, (const SampleParams*)s->smp_dev,
                      s->kc, s->vc, (int)s->max_seq, 0};
        yrow[i] = s->logits;
    }
    const GrpLayout L = grp_layout(m, n);
    int rc = CW_OK;
    if (cudaMalloc(&g->rows, n * sizeof(GrpRow)) != cudaSuccess ||
        cudaMalloc(&g->mem, L.total) != cudaSuccess)
        rc = set_error(CW_ERR_OOM, "cw_group_create: device allocation failed");
    if (rc == CW_OK &&
        (cudaMemsetAsync(g->mem, 0, L.total, ctx->stream) != cudaSuccess ||
         cudaMemcpyAsync(g->rows, h.data(), n * sizeof(GrpRow), cudaMemcpyHostToDevice,
                         ctx->stream) != cudaSuccess ||
         cudaMemcpyAsync((uint8_t*)g->mem + L.yrow, yrow.data(), n * sizeof(float*),
                         cudaMemcpyHostToDevice, ctx->stream) != cudaSuccess ||
         cudaMemcpyAsync((uint8_t*)g->mem + L.keys, keys.data(), n * 8, cudaMemcpyHostToDevice,
                         ctx->stream) != cudaSuccess ||
         cudaStreamSynchronize(ctx->stream) != cudaSuccess))
        rc = set_error(CW_ERR_CUDA, "cw_group_create: upload failed");
    if (rc != CW_OK) {
        cw_group_free(g);
        return rc;
    }
    *out = g;
    return CW_OK;
}

int cw_group_free(cw_group* g) {
    if (!g) return CW_OK;
    cudaSetDevice(g->m->ctx->device);
    cudaStreamSynchronize(g->m->ctx->stream);
    if (g->graph) cudaGraphExecDestroy(g->graph);
    if (g->rows) cudaFree(g->rows);
    if (g->mem) cudaFree(g->mem);
    delete g;
    return CW_OK;
}

int cw_group_set_streaming(cw_group* g, int on, int* streaming) {
    clear_error();
    CW_CHECK(g, CW_ERR_INVALID_ARG, "cw_group_set_streaming: group is NULL");
    CW_CHECK(on >= -1 && on <= 2, CW_ERR_INVALID_ARG, "cw_group_set_streaming: on must be -1..2");
    const int cur = g->streaming ? (g->mma ? 1 : 2) : 0;
    if (on >= 0 && on != cur) {
        cw_ctx* ctx = g->m->ctx;
        cudaSetDevice(ctx->device);
        CW_CHECK(!on || grp_streaming_ok(g->m, g->ss.size()), CW_ERR_UNSUPPORTED,
                 "cw_group_set_streaming: the group does not qualify for the streaming step");
        CW_TRY(on ? model_tile_weights(g->m) : model_pack_weights(g->m));
        CW_CUDA(cudaStreamSynchronize(ctx->stream));
        if (g->graph) cudaGraphExecDestroy(g->graph);
        g->graph = nullptr;
        g->streaming = on != 0;
        g->mma = on != 2;
    }
    if (streaming) *streaming = g->streaming ? (g->mma ? 1 : 2) : 0;
    return CW_OK;
}

int cw_group_run(cw_group* g, size_t n_steps) {
    clear_error();
    CW_CHECK(g, CW_ERR_INVALID_ARG, "cw_group_run: group is NULL");
    for (cw_session* s : g->ss)
        CW_CHECK(s->n_prompt > 0, CW_ERR_INVALID_ARG, "cw_group_run: a session has not begun");
    cudaSetDevice(g->m->ctx->device);
    for (size_t i = 0; i < n_steps; i++) CW_TRY(grp_step(g));
    CW_TRY(grp_sync(g));
    return check_device_status(g->m->ctx);
}

int cw_group_run_timed(cw_group* g, size_t n_steps, double* ms) {
    clear_error();
    CW_CHECK(g && ms, CW_ERR_INVALID_ARG, "cw_group_run_timed: bad arguments");
    cw_ctx* ctx = g->m->ctx;
    cudaSetDevice(ctx->device);
    cudaEvent_t e0, e1;
    CW_CUDA(cudaEventCreate(&e0));
    CW_CUDA(cudaEventCreate(&e1));
    int rc = CW_OK;
    if (!g->graph && n_steps) rc = grp_step(g), n_steps--;  // capture outside the timed region
    cudaEventRecord(e0, ctx->stream);
    for (size_t i = 0; i < n_steps && rc == CW_OK; i++) rc = grp_step(g);
    cudaEventRecord(e1, ctx->stream);
    cudaEventSynchronize(e1);
    float f = 0.f;
    cudaEventElapsedTime(&f, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    CW_TRY(rc);
    *ms = f;
    CW_TRY(grp_sync(g));
    return check_device_status(ctx);
}

}  // extern "C"
