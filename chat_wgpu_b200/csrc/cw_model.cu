// cw_model.cu -- the model layer of chat-wgpu (src/model/{mod,qwen3,layers,
// cache}.rs) on B200: GGUF load with Q4_0 weights kept Q4_0 in HBM, a decode
// session (KV cache + per-token device state), and one decode step built from
// five fused kernels per layer, replayed as a CUDA graph.
//
// Per token (src/model/qwen3.rs:139-191 composition):
//   embed        hidden = dequant(token_embd[token])            (qwen3.rs:128-133)
//   per layer
//     attn_in    x = rmsnorm(hidden); qkv = [Wq;Wk;Wv] x (+bias)  (:149-152)
//     attn       q/k = rmsnorm per head (QK-norm), RoPE, K/V row written at
//                pos, split-KV attention over pos+1 keys        (:154-177)
//     attn_out   hidden += Wo attn                              (:178-179)
//     ffn_in     x = rmsnorm(hidden); act = swiglu(Wg x, Wu x)  (:182-185)
//     ffn_out    hidden += Wd act                               (:186-187)
//   head         x = rmsnorm(hidden); logits = Wlm x; argmax    (:190, mod.rs:95-103)
//   finalize     next input = prompt[pos+1] or the argmax; pos += 1  (mod.rs:114-122)
// Families with post-norms (gemma2) defer each residual add into the next
// kernel's prologue so that no kernel reads the vector another CTA writes.
// Position, input token and the argmax live in device memory, so the same
// graph replays for every token.
#include <string.h>

#include <algorithm>
#include <cmath>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "cw_attn.cuh"
#include "cw_common.h"
#include "cw_device.cuh"
#include "cw_gemv.cuh"
#include "cw_gguf.h"
#include "cw_kquant.cuh"
#include "cw_ops.h"
#include "cw_model.h"
#include "cw_nccl.h"
#include "cw_q4.h"
#include "cw_tp_p2p.h"

namespace cw {

// ===========================================================================
// fused kernels
// ===========================================================================
// The prologue/epilogue vocabulary and argument block are shared with the
// streaming GEMV (cw_gemv.cuh); k_fgemv below is the fallback for K that the
// streaming kernel does not take (K/32 not a multiple of 8).
using FArgs = GemvArgs;

__device__ __forceinline__ float cta_sum(float v, float* red) {
    v = warp_sum(v);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }  // glu.wgsl:25
__device__ __forceinline__ float gelu_f(float x) {                                 // glu.wgsl:27-30
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ constexpr size_t fgemv_smem(int pro, int K) {
    return align_up(q24_bytes(K / 32), 16) + (pro == PRO_NORM ? (size_t)K * 4 : 0);
}

template <int PRO, int EPI, int R>
__global__ void __launch_bounds__(256) k_fgemv(FArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float red[8];
    __shared__ unsigned long long red_key[8];
    const int nb = a.K / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    Q24 s = q24_carve(smem, nb);
    const long groups = ((long)a.N + 8 * R - 1) / (8 * R);
    pdl_trigger();
    if (threadIdx.x == 0) {  // this CTA's weight rows do not depend on the predecessor
        for (long g = blockIdx.x; g < groups; g += gridDim.x) {
            long r0 = g * 8 * R, r1 = min((long)a.N, r0 + 8 * R);
            prefetch_l2(a.payload + (size_t)r0 * nb * 16, a.payload + (size_t)r1 * nb * 16);
            const __half* sc = reinterpret_cast<const __half*>(a.scales);
            prefetch_l2(sc + (size_t)r0 * nb, sc + (size_t)r1 * nb);
        }
    }
    pdl_wait();
    if (PRO == PRO_X) {
        q24_prepare<LAYOUT_GGUF>(s, a.x);
    } else {
        float* hbuf = reinterpret_cast<float*>(smem + align_up(q24_bytes(nb), 16));
        const int K = a.K;
        float inv_d = 0.f;
        if (a.delta && a.post_w) {
            float ss = 0.f;
            for (int i = threadIdx.x; i < K; i += blockDim.x) ss = fmaf(a.delta[i], a.delta[i], ss);
            ss = cta_sum(ss, red);
            inv_d = 1.0f / sqrtf(ss / (float)K + a.eps);
        }
        float ssh = 0.f;
        const bool wr = a.h_out && blockIdx.x == 0;
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            float h = a.base[i];
            if (a.delta) {
                float dv = a.delta[i];
                if (a.post_w) {
                    float gw = a.unit ? 1.0f + a.post_w[i] : a.post_w[i];
                    dv = __fmul_rn(__fmul_rn(dv, inv_d), gw);
                }
                h = h + dv;
            }
            hbuf[i] = h;
            if (wr) a.h_out[i] = h;
            ssh = fmaf(h, h, ssh);
        }
        ssh = cta_sum(ssh, red);
        const float inv = 1.0f / sqrtf(ssh / (float)K + a.eps);
        const bool wx = a.xn_out && blockIdx.x == 0;
        for (int b = warp; b < nb; b += (blockDim.x >> 5)) {
            int i = b * 32 + lane;
            float gw = a.unit ? 1.0f + a.norm_w[i] : a.norm_w[i];
            float v = __fmul_rn(__fmul_rn(hbuf[i], inv), gw);
            if (wx) a.xn_out[i] = v;
            q24_block<LAYOUT_GGUF>(s, b, v, lane);
        }
    }
    __syncthreads();

    unsigned long long best = argmax_key_init();
    for (long g = blockIdx.x; g < groups; g += gridDim.x) {
        long row0 = (g * 8 + warp) * R;
        if (row0 >= a.N) continue;
        float acc[R];
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = 0.f;
        q4_rows_dot<LAYOUT_GGUF, R>(s, a.payload, a.scales, row0, a.N, lane, acc);
#pragma unroll
        for (int r = 0; r < R; r++) acc[r] = warp_sum(acc[r]);
        if (EPI == EPI_GLU) {
            // interleaved rows: 2i = gate_i, 2i+1 = up_i
#pragma unroll
            for (int p = 0; p < R / 2; p++) {
                long row = row0 + 2 * p;
                if (lane == p && row < a.N) {
                    float gv = acc[2 * p], uv = acc[2 * p + 1];
                    float act = a.geglu ? gelu_f(gv) : silu_f(gv);
                    a.y[row / 2] = act * uv;
                }
            }
        } else if (EPI == EPI_HEAD) {
#pragma unroll
            for (int r = 0; r < R; r++) {
                long row = row0 + r;
                if (row < a.N) {
                    float v = acc[r];
                    if (a.softcap > 0.f) v = a.softcap * tanhf(v / a.softcap);
                    if (lane == r) a.y[row] = v;
                    unsigned long long k = argmax_key(v, (unsigned)row + a.key_offset);
                    best = k > best ? k : best;
                }
            }
        } else {
#pragma unroll
            for (int r = 0; r < R; r++) {
                long row = row0 + r;
                if (lane == r && row < a.N) {
                    if (EPI == EPI_RESID)
                        a.y[row] = a.y[row] + acc[r];
                    else
                        a.y[row] = a.bias ? acc[r] + a.bias[row] : acc[r];
                }
            }
        }
    }
    if (EPI == EPI_HEAD) {
        if (lane == 0) red_key[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = red_key[w] > best ? red_key[w] : best;
            atomicMax(a.key, best);
        }
    }
}

// ---- attention with QK-norm + RoPE + KV write fused in front -------------
struct AArgs {
    const float* qkv;      // [qd | kvd | kvd] raw projections
    const float* q_norm;   // QK-norm gains (qwen3.rs:154-155) or null
    const float* k_norm;
    float eps;
    const float* inv_freq; // RoPE table
    float* kc;             // this layer's cache [n_kv][max_seq][hd]
    float* vc;
    int max_seq;
    float* out;            // [n_heads * hd]
    float* part;
    unsigned* counters;
    int n_heads, n_kv, hd, n_splits, window;
    float scale, softcap;
    const DevState* st;
    float* q_out;  // optional: the normed, rotated q rows (hook tap "q")
};

// Warps of the per-stage attention CTA (4 keys each per pass): 16, or 8 for
// the variants whose per-lane state (EPL x GMAX) would not fit 128 registers.
template <int EPL, int GMAX>
constexpr int fa_nw() { return EPL * GMAX <= 16 ? 16 : 8; }

template <int EPL, int GMAX>
__global__ void __launch_bounds__(fa_nw<EPL, GMAX>() * 32) k_fattn(AArgs a) {
    constexpr int FA_NW = fa_nw<EPL, GMAX>();
    extern __shared__ float sm[];
    const int G = a.n_heads / a.n_kv, hd = a.hd;
    const int g = blockIdx.y, split = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    // The position is written by the previous step's finalize kernel, which an
    // early-launched chain of dependents can overtake: read it only after the
    // dependency wait (no global data read before pdl_wait may come from an
    // earlier kernel).
    pdl_wait();
    const int pos = a.st->pos, seq = pos + 1;
    const int n_active = attn_active_splits(attn_span(seq, a.window), a.n_splits);
    if (split >= n_active) return;
    int jlo, jhi;
    attn_range(seq, a.window, split, n_active, &jlo, &jhi);
    const bool holds = pos >= jlo && pos < jhi;
    if (threadIdx.x == 0) {  // cached rows [jlo, min(jhi, pos)) into L2 in one go
        int j1 = min(jhi, pos);
        if (j1 > jlo) {
            const float* kb0 = a.kc + ((size_t)g * a.max_seq) * hd;
            const float* vb0 = a.vc + ((size_t)g * a.max_seq) * hd;
            prefetch_l2(kb0 + (size_t)jlo * hd, kb0 + (size_t)j1 * hd);
            prefetch_l2(vb0 + (size_t)jlo * hd, vb0 + (size_t)j1 * hd);
        }
    }
    float* qs = sm + attn_smem_floats(G, hd, a.n_splits, FA_NW);  // [G][hd]
    float* ks = qs + (size_t)G * hd;           // [hd]
    const int qd = a.n_heads * hd, kvd = a.n_kv * hd;
    const int nrows = G + (holds ? 1 : 0);
    for (int r = warp; r < nrows; r += FA_NW) {
        const bool isq = r < G;
        const float* src = isq ? a.qkv + (size_t)(g * G + r) * hd : a.qkv + qd + (size_t)g * hd;
        const float* nw = isq ? a.q_norm : a.k_norm;
        float* dst = isq ? qs + (size_t)r * hd : ks;
        float v[EPL];
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            int d = lane + 32 * e;
            v[e] = d < hd ? src[d] : 0.f;
            ss = fmaf(v[e], v[e], ss);
        }
        if (nw) {  // norm.wgsl:20-37 over one head row
            ss = warp_sum(ss);
            float inv = 1.0f / sqrtf(ss / (float)hd + a.eps);
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                int d = lane + 32 * e;
                if (d < hd) v[e] = __fmul_rn(__fmul_rn(v[e], inv), nw[d]);
            }
        }
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            int d = lane + 32 * e;
            if (d < hd) dst[d] = v[e];
        }
    }
    __syncthreads();
    // RoPE (rope.wgsl:25-34) in place, one thread per rotated pair
    const int half = hd / 2;
    for (int i = threadIdx.x; i < nrows * half; i += blockDim.x) {
        int r = i / half, k = i - r * half;
        float* row = r < G ? qs + (size_t)r * hd : ks;
        float freq = __fmul_rn((float)pos, a.inv_freq[k]);
        float sn, cs;
        sincosf(freq, &sn, &cs);
        float lo = row[k], hi = row[k + half];
        row[k] = __fsub_rn(__fmul_rn(lo, cs), __fmul_rn(hi, sn));
        row[k + half] = __fadd_rn(__fmul_rn(hi, cs), __fmul_rn(lo, sn));
    }
    __syncthreads();
    if (a.q_out && split == 0)
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x) a.q_out[(size_t)g * G * hd + i] = qs[i];
    float* kbase = a.kc + (size_t)g * a.max_seq * hd;
    float* vbase = a.vc + (size_t)g * a.max_seq * hd;
    if (holds) {  // cache.rs:21-24: this token's K (normed, roped) and V at pos
        const float* vsrc = a.qkv + qd + kvd + (size_t)g * hd;
        for (int d = threadIdx.x; d < hd; d += blockDim.x) {
            kbase[(size_t)pos * hd + d] = ks[d];
            vbase[(size_t)pos * hd + d] = vsrc[d];
        }
    }
    __syncthreads();
    float* res = sm + FA_NW * G * (hd + 2);
    float* cwt = sm + (FA_NW + 1) * G * (hd + 2);
    attn_core<EPL, GMAX, KV_PLAIN, FA_NW>(qs, G, hd, kbase, vbase, hd, jlo, jhi, a.scale, a.softcap, sm,
                                   res);
    attn_finish(res, G, hd, g, split, n_active, a.n_splits, a.part, a.counters, a.out, cwt);
}

// ---- embed / finalize ------------------------------------------------------
// qwen3.rs:128-133: row `token` of token_embd, exact Q4_0 dequantisation.
__global__ void k_embed(const uint8_t* __restrict__ payload, const __half* __restrict__ scales,
                        int type, int dim, float scale, const DevState* __restrict__ st,
                        float* __restrict__ hidden) {
    pdl_trigger();
    pdl_wait();
    const unsigned tok = st->token;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float v = embed_elem(payload, scales, type, tok, dim, i);
        hidden[i] = scale > 0.f ? __fmul_rn(v, scale) : v;
    }
}

// Projections and LM heads kept as raw GGUF k-quant blocks (Q4_K / Q5_K /
// Q6_K: real checkpoints keep the LM head, and Q4_K_M files some projections,
// in these types).  Prologue: x = rmsnorm(h) (h = base, or base + delta,
// post-normed when post_w is set; CTA 0 writes h_out and xn_out) or x from
// global memory, staged once per CTA in shared memory.  Then one warp per
// output row (kq_dot: exact per-weight dequantisation, f32 accumulation) and
// the Q4_0 GEMV's epilogues: store (+bias), residual add, the gated unit over
// interleaved gate/up rows, or the LM head's soft-cap, logits and argmax key
// (atomicMax, ties -> lowest index).
template <int T, int PRO, int EPI>
__global__ void __launch_bounds__(256) k_kq_fgemv(FArgs a) {
    extern __shared__ float xs[];
    __shared__ float red[32];
    __shared__ unsigned long long red_key[8];
    constexpr int BYTES = KQ<T>::BYTES;
    const int K = a.K, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    pdl_wait();
    if (PRO == PRO_NORM) {
        float inv_d = 0.f;
        if (a.delta && a.post_w) {
            float ss = 0.f;
            for (int i = threadIdx.x; i < K; i += blockDim.x) ss = fmaf(a.delta[i], a.delta[i], ss);
            ss = cta_sum(ss, red);
            inv_d = 1.0f / sqrtf(ss / (float)K + a.eps);
        }
        float ssh = 0.f;
        const bool wh = a.h_out && blockIdx.x == 0;
        // loads of GEMV_PB elements issued before their math and stores
        for (int i0 = threadIdx.x; i0 < K; i0 += GEMV_PB * blockDim.x) {
            float hv[GEMV_PB], dv[GEMV_PB], gv[GEMV_PB];
#pragma unroll
            for (int u = 0; u < GEMV_PB; u++) {
                const int i = i0 + u * blockDim.x;
                const bool in = i < K;
                hv[u] = in ? a.base[i] : 0.f;
                dv[u] = in && a.delta ? a.delta[i] : 0.f;
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
                xs[i] = h;
                if (wh) a.h_out[i] = h;
                ssh = fmaf(h, h, ssh);
            }
        }
        ssh = cta_sum(ssh, red);
        const float inv = 1.0f / sqrtf(ssh / (float)K + a.eps);
        for (int i = threadIdx.x; i < K; i += blockDim.x) {
            const float gw = a.unit ? 1.0f + a.norm_w[i] : a.norm_w[i];
            const float v = __fmul_rn(__fmul_rn(xs[i], inv), gw);
            xs[i] = v;
            if (a.xn_out && blockIdx.x == 0) a.xn_out[i] = v;
        }
    } else {
        for (int i = threadIdx.x; i < K; i += blockDim.x) xs[i] = a.x[i];
    }
    __syncthreads();
    const int nbk = K / 256;
    auto dot = [&](int r) {  // KQ_UNROLL super-blocks' loads in flight at once
        const uint8_t* row = a.payload + (size_t)r * nbk * BYTES;
        float acc = 0.f;
        int b = 0;
        for (; b + KQ_UNROLL <= nbk; b += KQ_UNROLL) {
            KqRaw<T> raw[KQ_UNROLL];
#pragma unroll
            for (int u = 0; u < KQ_UNROLL; u++) raw[u] = kq_load<T>(row + (size_t)(b + u) * BYTES, lane);
#pragma unroll
            for (int u = 0; u < KQ_UNROLL; u++) acc = kq_dot<T>(raw[u], xs + 256 * (b + u), lane, acc);
        }
        for (; b < nbk; b++)
            acc = kq_dot<T>(kq_load<T>(row + (size_t)b * BYTES, lane), xs + 256 * b, lane, acc);
        return warp_sum(acc);
    };
    if (EPI == EPI_GLU) {  // rows 2i = gate_i, 2i+1 = up_i
        for (int i = blockIdx.x * 8 + warp; i < a.N / 2; i += gridDim.x * 8) {
            const float gv = dot(2 * i), uv = dot(2 * i + 1);
            if (lane == 0) a.y[i] = (a.geglu ? gelu_ref_f(gv) : silu_ref_f(gv)) * uv;
        }
        return;
    }
    unsigned long long best = argmax_key_init();
    for (int r = blockIdx.x * 8 + warp; r < a.N; r += gridDim.x * 8) {
        float v = dot(r);
        if (EPI == EPI_HEAD) {
            if (a.softcap > 0.f) v = a.softcap * tanhf(v / a.softcap);
            if (lane == 0) a.y[r] = v;
            const unsigned long long k = argmax_key(v, (unsigned)r + a.key_offset);
            best = k > best ? k : best;
        } else if (EPI == EPI_RESID) {
            if (lane == 0) a.y[r] = a.y[r] + v;
        } else {
            if (lane == 0) a.y[r] = a.bias ? v + a.bias[r] : v;
        }
    }
    if (EPI == EPI_HEAD) {
        if (lane == 0) red_key[warp] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int w = 1; w < (int)(blockDim.x >> 5); w++)
                best = red_key[w] > best ? red_key[w] : best;
            best = red_key[0] > best ? red_key[0] : best;
            atomicMax(a.key, best);
        }
    }
}

// mod.rs:114-122: the next input is the next prompt token while the prompt
// lasts, else the argmax, which is also appended to the output.
// n_ar: the tensor-parallel peer all-reduces this step ran (cw_tp_p2p.cu).
__global__ void k_finalize(DevState* st, const unsigned* __restrict__ prompt,
                           unsigned* __restrict__ toks, int decode, unsigned n_ar) {
    pdl_trigger();
    pdl_wait();
    int pos = st->pos;
    unsigned next;
    if (pos + 1 < st->n_prompt) {
        next = prompt[pos + 1];
    } else {
        unsigned tok = decode ? argmax_key_index(st->key) : 0u;
        toks[st->n_produced] = tok;
        st->n_produced = st->n_produced + 1;
        next = tok;
    }
    st->key = argmax_key_init();
    st->token = next;
    st->pos = pos + 1;
    st->ar_seq += n_ar;
}

__global__ void k_begin(DevState* st, const unsigned* __restrict__ prompt, int n_prompt,
                        const unsigned long long* __restrict__ bar) {
    st->pos = 0;
    st->token = prompt[0];
    st->n_prompt = n_prompt;
    st->n_produced = 0;
    st->key = argmax_key_init();
    st->bar_base = bar[0];  // the persistent step's counters continue from here
    st->ctr_base = bar[1];
    st->done = 0;
    st->stopped = 0;
    st->stall_us = 0;
}

// ---- hook taps (src/model/mod.rs:155-165) -----------------------------------
// Copy a tapped vector into slot pos % cap of its ring.
__global__ void k_tap(const float* __restrict__ src, int len, float* __restrict__ ring, int cap,
                      const DevState* __restrict__ st) {
    float* dst = ring + (size_t)(st->pos % cap) * len;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < len; i += gridDim.x * blockDim.x)
        dst[i] = src[i];
}
// Post-norm families: the residual sum base + rmsnorm(delta) * gain(w) that
// the next kernel's prologue forms, computed into the ring for a tap.
__global__ void k_tap_postadd(const float* __restrict__ base, const float* __restrict__ delta,
                              const float* __restrict__ w, int unit, float eps, int dim,
                              float* __restrict__ ring, int cap, const DevState* __restrict__ st) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(delta[i], delta[i], ss);
    const float inv = 1.0f / sqrtf(cta_sum(ss, red) / (float)dim + eps);
    float* dst = ring + (size_t)(st->pos % cap) * dim;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        const float gw = unit ? 1.0f + w[i] : w[i];
        dst[i] = base[i] + __fmul_rn(__fmul_rn(delta[i], inv), gw);
    }
}

// ===========================================================================
// host side
// ===========================================================================
// Kernel launch on the context stream; with ctx->pdl the launch carries
// programmatic stream serialisation so it may overlap its predecessor up to
// the kernel's pdl_wait().
template <typename... KArgs, typename... Args>
static int launch_k(cw_ctx* ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                    Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ctx->pdl ? 1 : 0;
    CW_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
    return CW_OK;
}

template <int PRO, int EPI, int R>
static int launch_fgemv(cw_ctx* ctx, const FArgs& a) {
    size_t smem = fgemv_smem(PRO, a.K);
    auto kern = k_fgemv<PRO, EPI, R>;
    if (smem > 48 * 1024) {
        CW_CHECK((int)smem <= ctx->max_smem_optin, CW_ERR_UNSUPPORTED,
                 "fused gemv: K=%d needs %zu bytes of shared memory", a.K, smem);
        CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    }
    int per_sm = 0;
    CW_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem));
    per_sm = std::max(per_sm, 1);
    long groups = ((long)a.N + 8 * R - 1) / (8 * R);
    long grid = std::min<long>(groups, (long)ctx->sm_count * per_sm);
    CW_TRY(launch_k(ctx, kern, dim3((unsigned)grid), dim3(256), smem, a));
    return check_launch("fused gemv");
}

// Rows per warp for a GEMV of N rows: enough warps to cover every SM twice.
static int pick_r(cw_ctx* ctx, long N) {
    long sm2 = 2L * ctx->sm_count * 8;
    if (N >= sm2 * 4) return 4;
    if (N >= sm2 * 2) return 2;
    return 1;
}

template <int PRO, int EPI>
static int fgemv(cw_ctx* ctx, const FArgs& a) {
    if (sgemv_supported(LAYOUT_GGUF, a.K)) return launch_sgemv(ctx, LAYOUT_GGUF, PRO, EPI, a, ctx->pdl);
    int r = pick_r(ctx, a.N);
    if (r == 4) return launch_fgemv<PRO, EPI, 4>(ctx, a);
    if constexpr (EPI == EPI_GLU) {
        return launch_fgemv<PRO, EPI, 2>(ctx, a);  // gate/up rows come in pairs
    } else {
        if (r == 2) return launch_fgemv<PRO, EPI, 2>(ctx, a);
        return launch_fgemv<PRO, EPI, 1>(ctx, a);
    }
}

template <int T, int PRO, int EPI>
static int kq_fgemv_t(cw_ctx* ctx, const FArgs& a) {
    auto kern = k_kq_fgemv<T, PRO, EPI>;
    const size_t smem = (size_t)a.K * 4;
    if (smem > 48 * 1024) {
        CW_CHECK((int)smem <= ctx->max_smem_optin, CW_ERR_UNSUPPORTED,
                 "k-quant gemv: K=%d needs %zu bytes of shared memory", a.K, smem);
        CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    }
    // as many CTAs as fit on the SMs at once: each warp's rows are latency-bound
    int per_sm = 0;
    CW_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem));
    const long rows = EPI == EPI_GLU ? a.N / 2 : a.N;
    const int grid =
        (int)std::min<long>((rows + 7) / 8, (long)ctx->sm_count * std::max(per_sm, 1));
    CW_TRY(launch_k(ctx, kern, dim3(grid), dim3(256), smem, a));
    return check_launch("k-quant gemv");
}

// Q4_K / Q5_K projections the streaming GEMV takes (the gated unit needs two
// rows per chunk: K <= 12288).
template <int EPI>
static bool kq_stream_ok(int K) {
    return sgemv_supported(LAYOUT_Q4K, K) && (EPI != EPI_GLU || K / 32 <= GemvC384::NB_MAX);
}

// One projection of the per-stage step over weight `w`: the streaming GEMV
// (Q4_0 planes, raw Q4_K / Q5_K super-blocks, the Q6_K split), or the
// per-row GEMV for the other raw types.
template <int PRO, int EPI>
static int proj(cw_ctx* ctx, const QW& w, FArgs a) {
    a.payload = w.payload;
    a.scales = w.scales;
    a.K = w.in_f;
    a.N = w.rows;
    switch (w.type) {
        case GGML_Q4_0: return fgemv<PRO, EPI>(ctx, a);
        case GGML_Q4_K:
            if (kq_stream_ok<EPI>(a.K)) return launch_sgemv(ctx, LAYOUT_Q4K, PRO, EPI, a, ctx->pdl);
            return kq_fgemv_t<GGML_Q4_K, PRO, EPI>(ctx, a);
        case GGML_Q5_K:
            if (kq_stream_ok<EPI>(a.K)) return launch_sgemv(ctx, LAYOUT_Q5K, PRO, EPI, a, ctx->pdl);
            return kq_fgemv_t<GGML_Q5_K, PRO, EPI>(ctx, a);
        case GGML_Q6_K:
            if (w.split && kq_stream_ok<EPI>(a.K)) {
                a.payload = w.split;
                a.scales = w.split_d;
                return launch_sgemv(ctx, LAYOUT_Q6K, PRO, EPI, a, ctx->pdl);
            }
            return kq_fgemv_t<GGML_Q6_K, PRO, EPI>(ctx, a);
        case GGML_F32: return kq_fgemv_t<GGML_F32, PRO, EPI>(ctx, a);
        case GGML_F16: return kq_fgemv_t<GGML_F16, PRO, EPI>(ctx, a);
        case GGML_BF16: return kq_fgemv_t<GGML_BF16, PRO, EPI>(ctx, a);
        case GGML_Q8_0:
            if (w.split && kq_stream_ok<EPI>(a.K)) {
                a.payload = w.split;
                a.scales = w.split_d;
                return launch_sgemv(ctx, LAYOUT_Q8, PRO, EPI, a, ctx->pdl);
            }
            return kq_fgemv_t<GGML_Q8_0, PRO, EPI>(ctx, a);
        case GGML_Q4_1: return kq_fgemv_t<GGML_Q4_1, PRO, EPI>(ctx, a);
        default: return set_error(CW_ERR_UNSUPPORTED, "projection of ggml type %d", w.type);
    }
}

template <int EPL, int GM>
static int fattn_go(cw_ctx* ctx, const AArgs& a, dim3 grid) {
    constexpr int FA_NW = fa_nw<EPL, GM>();
    const size_t smem =
        (attn_smem_floats(a.n_heads / a.n_kv, a.hd, a.n_splits, FA_NW) +
         (size_t)(a.n_heads / a.n_kv) * a.hd + a.hd) * sizeof(float);
    if (smem > 48 * 1024)
        CW_CUDA(cudaFuncSetAttribute(k_fattn<EPL, GM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem));
    CW_TRY(launch_k(ctx, k_fattn<EPL, GM>, grid, dim3(FA_NW * 32), smem, a));
    return CW_OK;
}

template <int EPL>
static int launch_fattn_e(cw_ctx* ctx, const AArgs& a, dim3 grid) {
    int G = a.n_heads / a.n_kv;
#define CW_FATTN(GM) CW_TRY((fattn_go<EPL, GM>(ctx, a, grid)))
    if (G <= 1) CW_FATTN(1);
    else if (G <= 2) CW_FATTN(2);
    else if (G <= 4) CW_FATTN(4);
    else CW_FATTN(8);
#undef CW_FATTN
    return check_launch("fused attention");
}

static int launch_fattn(cw_ctx* ctx, const AArgs& a) {
    dim3 grid(a.n_splits, a.n_kv);
    int epl = (a.hd + 31) / 32;
    if (epl <= 1) return launch_fattn_e<1>(ctx, a, grid);
    if (epl <= 2) return launch_fattn_e<2>(ctx, a, grid);
    if (epl <= 4) return launch_fattn_e<4>(ctx, a, grid);
    return launch_fattn_e<8>(ctx, a, grid);
}

// ---- loading ----------------------------------------------------------------
static int dev_alloc(cw_model* m, size_t nbytes, void** p) {
    cw_buf b;
    BufEntry* e;
    CW_TRY(buf_new(m->ctx, nbytes, BUF_PERSISTENT, &b, &e));
    m->owned.push_back(b);
    *p = e->ptr;
    return CW_OK;
}

static float f16_bits_to_f32(uint16_t h) {
    // exact decode incl. subnormals / inf / nan (dequant.rs:9-21)
    int sign = (h >> 15) & 1, e = (h >> 10) & 0x1f;
    float mant = (float)(h & 0x3ff), mag;
    if (e == 0) mag = mant * ldexpf(1.0f, -24);
    else if (e == 0x1f) mag = mant == 0.f ? INFINITY : NAN;
    else mag = (1.0f + mant / 1024.0f) * ldexpf(1.0f, e - 15);
    return sign ? -mag : mag;
}

static int load_vec(cw_model* m, const GgufFile& f, const std::string& name, size_t len,
                    float** out) {
    const GgufTensor* t = f.tensor(name);
    CW_CHECK(t, CW_ERR_NOT_FOUND, "missing tensor %s", name.c_str());
    CW_CHECK(t->n_elems == len, CW_ERR_FORMAT, "tensor %s has %llu elements, expected %zu",
             name.c_str(), (unsigned long long)t->n_elems, len);
    std::vector<float> h(len);
    if (t->type == GGML_F32) {
        memcpy(h.data(), t->data, len * 4);
    } else if (t->type == GGML_F16) {
        const uint16_t* s = (const uint16_t*)t->data;
        for (size_t i = 0; i < len; i++) h[i] = f16_bits_to_f32(s[i]);
    } else if (t->type == GGML_BF16) {
        const uint16_t* s = (const uint16_t*)t->data;
        for (size_t i = 0; i < len; i++) {
            uint32_t u = (uint32_t)s[i] << 16;
            memcpy(&h[i], &u, 4);
        }
    } else {
        return set_error(CW_ERR_UNSUPPORTED, "vector %s has type %s (F32/F16/BF16 expected)",
                         name.c_str(), ggml_type_name(t->type));
    }
    void* p;
    CW_TRY(dev_alloc(m, len * 4, &p));
    // stream-ordered with the kernels that read it (the context stream does
    // not wait for the legacy default stream) and complete before h dies
    CW_CUDA(cudaMemcpyAsync(p, h.data(), len * 4, cudaMemcpyHostToDevice, m->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(m->ctx->stream));
    *out = (float*)p;
    return CW_OK;
}

// Q6_K / Q8_0 weight: add the aligned split the streaming decode GEMV reads
// (same bytes as the raw blocks: payload plane, then the f16 d plane).
static int add_stream_split(cw_model* m, QW* w) {
    if (w->type == GGML_Q8_0 && sgemv_supported(LAYOUT_Q8, w->in_f)) {
        const size_t nb = (size_t)w->rows * (w->in_f / 32);
        void* p = nullptr;
        CW_TRY(dev_alloc(m, nb * 34, &p));
        uint8_t* base = (uint8_t*)p;
        CW_TRY(q8_split(m->ctx, w->payload, nb, base, (__half*)(base + nb * 32)));
        CW_CUDA(cudaStreamSynchronize(m->ctx->stream));
        w->split = base;
        w->split_d = (const __half*)(base + nb * 32);
        return CW_OK;
    }
    if (w->type != GGML_Q6_K || !sgemv_supported(LAYOUT_Q6K, w->in_f)) return CW_OK;
    const size_t nsb = (size_t)w->rows * (w->in_f / 256);
    void* p = nullptr;
    CW_TRY(dev_alloc(m, nsb * 210, &p));
    uint8_t* base = (uint8_t*)p;
    CW_TRY(q6k_split(m->ctx, w->payload, nsb, base, (__half*)(base + nsb * 208)));
    CW_CUDA(cudaStreamSynchronize(m->ctx->stream));
    w->split = base;
    w->split_d = (const __half*)(base + nsb * 208);
    return CW_OK;
}

// Load one or more Q4_0 [rows_i, in_f] tensors as a single packed weight.
// interleave: two parts with equal rows become rows p0[0], p1[0], p0[1], ...
// A token embedding or LM head stored as GGUF Q6_K (real Q4_0 checkpoints often
// keep these in Q6_K): the raw super-blocks go to HBM unchanged.
static int load_q6k(cw_model* m, const GgufTensor* t, size_t in_f, QW* out, int rdiv = 1,
                    int ridx = 0) {
    CW_CHECK(in_f % 256 == 0, CW_ERR_UNSUPPORTED,
             "tensor %s is Q6_K: its rows (%zu) must be a multiple of 256", t->name.c_str(), in_f);
    CW_CHECK(!t->dims.empty() && t->dims[0] == in_f && t->n_elems % in_f == 0, CW_ERR_FORMAT,
             "tensor %s: inner dimension %llu, expected %zu", t->name.c_str(),
             (unsigned long long)(t->dims.empty() ? 0 : t->dims[0]), in_f);
    const size_t rows = t->n_elems / in_f;
    CW_CHECK(t->nbytes == rows * (in_f / 256) * 210, CW_ERR_FORMAT, "tensor %s: %zu bytes",
             t->name.c_str(), t->nbytes);
    CW_CHECK(rows % rdiv == 0, CW_ERR_UNSUPPORTED, "tensor %s: %zu rows do not split %d ways",
             t->name.c_str(), rows, rdiv);
    // rows [ridx, ridx + 1) * rows / rdiv: a contiguous byte range of the raw blocks
    const size_t n = rows / rdiv, nbytes = t->nbytes / rdiv;
    void* p = nullptr;
    CW_TRY(dev_alloc(m, nbytes, &p));
    CW_CUDA(cudaMemcpyAsync(p, t->data + nbytes * ridx, nbytes, cudaMemcpyHostToDevice,
                            m->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(m->ctx->stream));
    out->payload = (const uint8_t*)p;
    out->scales = nullptr;
    out->rows = (int)n;
    out->in_f = (int)in_f;
    out->type = GGML_Q6_K;
    out->buf = m->owned.back();
    return add_stream_split(m, out);
}

// Q4_0 (packed planes) or Q6_K (raw), by the tensor's type.
static int load_q4_or_q6k(cw_model* m, const GgufFile& f, const std::string& name, size_t in_f,
                          QW* out);

static bool is_kquant(uint32_t t) { return t == GGML_Q4_K || t == GGML_Q5_K || t == GGML_Q6_K; }
// Types kept in HBM as the file's raw rows and read 256 weights at a time
// (cw_kquant.cuh): the k-quants and the other types the reference's loader
// dequantises (tensor_f32, gguf.rs:109-121: F32, F16, Q4_1, Q8_0), plus BF16
// (dequant_bf16, dequant.rs:41-43).
static bool is_raw(uint32_t t) {
    return is_kquant(t) || t == GGML_F32 || t == GGML_F16 || t == GGML_BF16 || t == GGML_Q8_0 ||
           t == GGML_Q4_1;
}

// Raw-type tensors `names` of one type kept as the file's rows, stacked by
// rows (or interleaved row by row: gate/up).
static int load_kq(cw_model* m, const GgufFile& f, const std::vector<std::string>& names,
                   size_t in_f, bool interleave, QW* out) {
    std::vector<const GgufTensor*> parts;
    for (auto& n : names) {
        const GgufTensor* t = f.tensor(n);
        CW_CHECK(t, CW_ERR_NOT_FOUND, "missing tensor %s", n.c_str());
        CW_CHECK(is_raw(t->type) && t->type == f.tensor(names[0])->type, CW_ERR_UNSUPPORTED,
                 "tensor %s is %s; expected %s", n.c_str(), ggml_type_name(t->type),
                 ggml_type_name(f.tensor(names[0])->type));
        CW_CHECK(in_f % 256 == 0 && !t->dims.empty() && t->dims[0] == in_f &&
                     t->n_elems % in_f == 0,
                 CW_ERR_FORMAT, "tensor %s: inner dimension must be %zu (a multiple of 256)",
                 n.c_str(), in_f);
        parts.push_back(t);
    }
    CW_CHECK(!interleave || (parts.size() == 2 && parts[0]->n_elems == parts[1]->n_elems),
             CW_ERR_FORMAT, "interleaved weights need two equal parts");
    const uint32_t type = parts[0]->type;
    const size_t rb = ggml_row_bytes(type, in_f);
    size_t rows = 0;
    for (auto* t : parts) {
        CW_CHECK(t->nbytes == t->n_elems / in_f * rb, CW_ERR_FORMAT, "tensor %s: %zu bytes",
                 t->name.c_str(), t->nbytes);
        rows += t->n_elems / in_f;
    }
    std::vector<uint8_t> stage(rows * rb);
    if (!interleave) {
        size_t off = 0;
        for (auto* t : parts) {
            memcpy(stage.data() + off, t->data, t->nbytes);
            off += t->nbytes;
        }
    } else {
        for (size_t r = 0; r < rows / 2; r++) {
            memcpy(stage.data() + (2 * r) * rb, parts[0]->data + r * rb, rb);
            memcpy(stage.data() + (2 * r + 1) * rb, parts[1]->data + r * rb, rb);
        }
    }
    void* p = nullptr;
    CW_TRY(dev_alloc(m, stage.size(), &p));
    CW_CUDA(cudaMemcpyAsync(p, stage.data(), stage.size(), cudaMemcpyHostToDevice,
                            m->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(m->ctx->stream));
    out->payload = (const uint8_t*)p;
    out->scales = nullptr;
    out->rows = (int)rows;
    out->in_f = (int)in_f;
    out->type = (int)type;
    out->buf = m->owned.back();
    m->info.weight_bytes += stage.size();
    return add_stream_split(m, out);
}

// One projection (or a stack / interleave of several) by the tensors' type:
// Q4_0 packed planes, or raw k-quant blocks.
static int load_proj(cw_model* m, const GgufFile& f, const std::vector<std::string>& names,
                     size_t in_f, bool interleave, QW* out);

// Q4_0 tensors `names` stacked by rows (or interleaved row by row), optionally
// sliced for tensor parallelism: rows [k/rdiv, (k+1)/rdiv) of each part with
// k = ridx, and the column blocks [c/cdiv, (c+1)/cdiv) with c = cidx.
static int load_q4_slice(cw_model* m, const GgufFile& f, const std::vector<std::string>& names,
                         size_t in_f, bool interleave, int rdiv, int ridx, int cdiv, int cidx,
                         QW* out);

static int load_q4(cw_model* m, const GgufFile& f, const std::vector<std::string>& names,
                   size_t in_f, bool interleave, QW* out) {
    std::vector<const GgufTensor*> parts;
    size_t rows = 0;
    const size_t rb = in_f / 32 * 18;
    for (auto& n : names) {
        const GgufTensor* t = f.tensor(n);
        CW_CHECK(t, CW_ERR_NOT_FOUND, "missing tensor %s", n.c_str());
        CW_CHECK(t->type == GGML_Q4_0, CW_ERR_UNSUPPORTED,
                 "tensor %s is %s; the decode path takes Q4_0 matrices", n.c_str(),
                 ggml_type_name(t->type));
        CW_CHECK(!t->dims.empty() && t->dims[0] == in_f && t->n_elems % in_f == 0, CW_ERR_FORMAT,
                 "tensor %s: inner dimension %llu, expected %zu", n.c_str(),
                 (unsigned long long)(t->dims.empty() ? 0 : t->dims[0]), in_f);
        parts.push_back(t);
        rows += t->n_elems / in_f;
    }
    CW_CHECK(!interleave || (parts.size() == 2 && parts[0]->n_elems == parts[1]->n_elems),
             CW_ERR_FORMAT, "interleaved weights need two equal parts");
    size_t nbytes = rows * rb;
    void* tmp = nullptr;
    CW_CUDA(cudaMalloc(&tmp, nbytes));
    cudaError_t ce = cudaSuccess;
    if (!interleave) {
        size_t off = 0;
        for (auto* t : parts) {
            ce = cudaMemcpyAsync((char*)tmp + off, t->data, t->nbytes, cudaMemcpyHostToDevice,
                                 m->ctx->stream);
            if (ce != cudaSuccess) break;
            off += t->nbytes;
        }
    } else {
        size_t r1 = parts[0]->n_elems / in_f;
        std::vector<uint8_t> stage(nbytes);
        for (size_t r = 0; r < r1; r++) {
            memcpy(stage.data() + (2 * r) * rb, parts[0]->data + r * rb, rb);
            memcpy(stage.data() + (2 * r + 1) * rb, parts[1]->data + r * rb, rb);
        }
        ce = cudaMemcpyAsync(tmp, stage.data(), nbytes, cudaMemcpyHostToDevice, m->ctx->stream);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(m->ctx->stream);  // before stage dies
    }
    if (ce != cudaSuccess) {
        cudaStreamSynchronize(m->ctx->stream);
        cudaFree(tmp);
        return set_error(CW_ERR_CUDA, "weight upload: %s", cudaGetErrorString(ce));
    }
    // the upload and the repack are ordered on the context stream: a plain
    // cudaMemcpy from pageable memory can return before its DMA lands, and
    // the non-blocking context stream would not wait for it
    cw_buf b;
    int rc = pack_q4_0(m->ctx, tmp, rows, in_f, &b);
    cudaStreamSynchronize(m->ctx->stream);
    cudaFree(tmp);
    CW_TRY(rc);
    m->owned.push_back(b);
    BufEntry& e = m->ctx->bufs[b];
    out->payload = (const uint8_t*)e.ptr;
    out->scales = (const __half*)((const char*)e.ptr + e.scale_off);
    out->rows = (int)rows;
    out->in_f = (int)in_f;
    out->buf = b;
    m->info.weight_bytes += rows * rb;
    return CW_OK;
}

static int load_q4_slice(cw_model* m, const GgufFile& f, const std::vector<std::string>& names,
                         size_t in_f, bool interleave, int rdiv, int ridx, int cdiv, int cidx,
                         QW* out) {
    const size_t nb = in_f / 32, rb = nb * 18;
    CW_CHECK(nb % cdiv == 0, CW_ERR_UNSUPPORTED, "%s: %zu blocks per row do not split %d ways",
             names[0].c_str(), nb, cdiv);
    const size_t cb0 = nb / cdiv * cidx, cbn = nb / cdiv, rbs = cbn * 18;
    std::vector<const GgufTensor*> parts;
    for (auto& n : names) {
        const GgufTensor* t = f.tensor(n);
        CW_CHECK(t, CW_ERR_NOT_FOUND, "missing tensor %s", n.c_str());
        CW_CHECK(t->type == GGML_Q4_0, CW_ERR_UNSUPPORTED,
                 "tensor %s is %s; the decode path takes Q4_0 matrices", n.c_str(),
                 ggml_type_name(t->type));
        CW_CHECK(!t->dims.empty() && t->dims[0] == in_f && t->n_elems % in_f == 0, CW_ERR_FORMAT,
                 "tensor %s: inner dimension %llu, expected %zu", n.c_str(),
                 (unsigned long long)(t->dims.empty() ? 0 : t->dims[0]), in_f);
        CW_CHECK((t->n_elems / in_f) % rdiv == 0, CW_ERR_UNSUPPORTED,
                 "tensor %s: %llu rows do not split %d ways", n.c_str(),
                 (unsigned long long)(t->n_elems / in_f), rdiv);
        parts.push_back(t);
    }
    CW_CHECK(!interleave || (parts.size() == 2 && parts[0]->n_elems == parts[1]->n_elems),
             CW_ERR_FORMAT, "interleaved weights need two equal parts");
    // the selected rows of every part, in output order
    std::vector<const uint8_t*> src;
    if (!interleave) {
        for (auto* t : parts) {
            const size_t n = t->n_elems / in_f / rdiv, r0 = n * ridx;
            for (size_t r = 0; r < n; r++) src.push_back(t->data + (r0 + r) * rb);
        }
    } else {
        const size_t n = parts[0]->n_elems / in_f / rdiv, r0 = n * ridx;
        for (size_t r = 0; r < n; r++) {
            src.push_back(parts[0]->data + (r0 + r) * rb);
            src.push_back(parts[1]->data + (r0 + r) * rb);
        }
    }
    const size_t rows = src.size();
    std::vector<uint8_t> stage(rows * rbs);
    for (size_t r = 0; r < rows; r++) memcpy(stage.data() + r * rbs, src[r] + cb0 * 18, rbs);
    void* tmp = nullptr;
    CW_CUDA(cudaMalloc(&tmp, stage.size()));
    cudaError_t ce = cudaMemcpyAsync(tmp, stage.data(), stage.size(), cudaMemcpyHostToDevice,
                                     m->ctx->stream);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(m->ctx->stream);
    if (ce != cudaSuccess) {
        cudaFree(tmp);
        return set_error(CW_ERR_CUDA, "weight upload: %s", cudaGetErrorString(ce));
    }
    cw_buf b;
    int rc = pack_q4_0(m->ctx, tmp, rows, cbn * 32, &b);
    cudaStreamSynchronize(m->ctx->stream);
    cudaFree(tmp);
    CW_TRY(rc);
    m->owned.push_back(b);
    BufEntry& e = m->ctx->bufs[b];
    out->payload = (const uint8_t*)e.ptr;
    out->scales = (const __half*)((const char*)e.ptr + e.scale_off);
    out->rows = (int)rows;
    out->in_f = (int)(cbn * 32);
    out->buf = b;
    m->info.weight_bytes += rows * rbs;
    return CW_OK;
}

static int load_proj(cw_model* m, const GgufFile& f, const std::vector<std::string>& names,
                     size_t in_f, bool interleave, QW* out) {
    const GgufTensor* t = f.tensor(names[0]);
    CW_CHECK(t, CW_ERR_NOT_FOUND, "missing tensor %s", names[0].c_str());
    if (is_raw(t->type)) {
        CW_CHECK(m->tp_world == 1, CW_ERR_UNSUPPORTED,
                 "tensor %s is %s; tensor parallelism takes Q4_0 projections", names[0].c_str(),
                 ggml_type_name(t->type));
        return load_kq(m, f, names, in_f, interleave, out);
    }
    return load_q4(m, f, names, in_f, interleave, out);
}

static int load_q4_or_q6k(cw_model* m, const GgufFile& f, const std::string& name, size_t in_f,
                          QW* out) {
    const GgufTensor* t = f.tensor(name);
    CW_CHECK(t, CW_ERR_NOT_FOUND, "missing tensor %s", name.c_str());
    if (t->type == GGML_Q6_K) return load_q6k(m, t, in_f, out);
    return load_q4(m, f, {name}, in_f, false, out);
}

static int model_load(cw_model* m, const std::string& path) {
    GgufFile f;
    std::string err;
    int rc = f.open(path, err);
    if (rc != CW_OK) return set_error(rc, "%s", err.c_str());
    std::string arch = f.meta_str("general.architecture");
    if (arch.empty()) arch = "qwen3";
    cw_model_info& I = m->info;
    snprintf(I.arch, sizeof I.arch, "%s", arch.c_str());
    int family;
    if (arch == "qwen3") family = 0;
    else if (arch == "qwen2" || arch == "llama") family = 1;
    else if (arch == "gemma2") family = 2;
    else return set_error(CW_ERR_UNSUPPORTED, "unsupported architecture '%s'", arch.c_str());
    auto K = [&](const char* s) { return arch + "." + s; };
    // qwen3.rs:45-53
    I.n_layers = f.meta_u32(K("block_count"));
    I.dim = f.meta_u32(K("embedding_length"));
    I.n_heads = f.meta_u32(K("attention.head_count"));
    I.n_kv = f.meta_u32(K("attention.head_count_kv"), I.n_heads);
    I.head_dim = f.meta_u32(K("attention.key_length"), I.n_heads ? I.dim / I.n_heads : 0);
    I.hidden = f.meta_u32(K("feed_forward_length"));
    I.eps = f.meta_f32(K("attention.layer_norm_rms_epsilon"), 1e-6f);
    I.rope_theta = f.meta_f32(K("rope.freq_base"), family == 2 ? 10000.f : 1000000.f);
    I.vocab = f.meta_u32(K("vocab_size"));
    if (!I.vocab) {  // gguf.rs:171-177
        if (const GgufTensor* te = f.tensor("token_embd.weight"))
            for (auto d : te->dims) I.vocab = std::max<uint32_t>(I.vocab, (uint32_t)d);
    }
    I.norm_kind = family == 2 ? 1 : 0;
    I.activation = family == 2 ? 1 : 0;
    I.qk_norm = family == 0 ? 1 : 0;
    I.post_norms = family == 2 ? 1 : 0;
    if (family == 2) {
        I.sliding_window = f.meta_u32(K("attention.sliding_window"));
        I.attn_softcap = f.meta_f32(K("attn_logit_softcapping"));
        I.final_softcap = f.meta_f32(K("final_logit_softcapping"));
        I.embed_scale = sqrtf((float)I.dim);
    }
    CW_CHECK(I.n_layers && I.dim && I.n_heads && I.n_kv && I.head_dim && I.hidden && I.vocab,
             CW_ERR_FORMAT, "model metadata incomplete");
    CW_CHECK(I.n_heads % I.n_kv == 0 && I.n_heads / I.n_kv <= 8, CW_ERR_UNSUPPORTED,
             "GQA group %u/%u not supported (n_kv | n_heads, group <= 8)", I.n_heads, I.n_kv);
    CW_CHECK(I.head_dim <= 256 && I.head_dim % 2 == 0, CW_ERR_UNSUPPORTED,
             "head_dim %u not supported (even, <= 256)", I.head_dim);
    CW_CHECK(I.dim % 32 == 0 && I.hidden % 32 == 0 && (I.n_heads * I.head_dim) % 32 == 0,
             CW_ERR_UNSUPPORTED, "dimensions must be multiples of 32");
    const size_t qd = (size_t)I.n_heads * I.head_dim, kvd = (size_t)I.n_kv * I.head_dim;
    // tensor parallelism over T ranks (Megatron-style): rank r holds heads
    // [r, r+1) * n_heads/T (with their KV heads) and FFN columns
    // [r, r+1) * hidden/T as row slices of q/k/v and gate/up and the matching
    // column slices of the O and down projections, whose partial outputs are
    // summed over the ranks; the LM head is split by vocabulary rows
    const int T = m->tp_world, r = m->tp_rank;
    if (T > 1)
        CW_CHECK(I.n_kv % T == 0 && I.hidden % (32 * T) == 0 && I.vocab % T == 0 &&
                     qd % (32 * T) == 0,
                 CW_ERR_UNSUPPORTED,
                 "tensor parallelism over %d ranks needs n_kv (%u), hidden/32 (%u), vocab (%u) "
                 "and q width/32 (%zu) divisible by %d",
                 T, I.n_kv, I.hidden / 32, I.vocab, qd / 32, T);
    m->vocab_full = I.vocab;
    m->L.resize(I.n_layers);
    for (uint32_t i = 0; i < I.n_layers; i++) {
        Layer& l = m->L[i];
        std::string p = "blk." + std::to_string(i) + ".";
        CW_TRY(load_vec(m, f, p + "attn_norm.weight", I.dim, &l.attn_norm));
        const std::vector<std::string> qkv = {p + "attn_q.weight", p + "attn_k.weight",
                                              p + "attn_v.weight"};
        uint32_t qt[3];
        for (int j = 0; j < 3; j++) {
            const GgufTensor* t = f.tensor(qkv[j]);
            CW_CHECK(t, CW_ERR_NOT_FOUND, "missing tensor %s", qkv[j].c_str());
            qt[j] = t->type;
        }
        if (qt[0] == qt[1] && qt[1] == qt[2]) {
            CW_TRY(T > 1 ? load_q4_slice(m, f, qkv, I.dim, false, T, r, 1, 0, &l.qkv)
                         : load_proj(m, f, qkv, I.dim, false, &l.qkv));
            CW_CHECK((size_t)l.qkv.rows == (qd + 2 * kvd) / T, CW_ERR_FORMAT,
                     "layer %u: q/k/v rows %d", i, l.qkv.rows);
        } else {  // mixed types: two or three weights over one qkv vector
            CW_CHECK(T == 1, CW_ERR_UNSUPPORTED,
                     "layer %u: q/k/v of different types; tensor parallelism takes Q4_0", i);
            l.qkv_split = true;
            // consecutive tensors of one type stack into one weight (one GEMV
            // launch): q+k | v, or q | k+v; slots left over keep 0 rows
            QW* dst[3] = {&l.q, &l.k, &l.v};
            for (int j = 0, slot = 0; j < 3; slot++) {
                int e = j + 1;
                while (e < 3 && qt[e] == qt[j]) e++;
                CW_TRY(load_proj(m, f, std::vector<std::string>(qkv.begin() + j, qkv.begin() + e),
                                 I.dim, false, dst[slot]));
                j = e;
            }
            CW_CHECK((size_t)(l.q.rows + l.k.rows + l.v.rows) == qd + 2 * kvd, CW_ERR_FORMAT,
                     "layer %u: q/k/v rows %d/%d/%d", i, l.q.rows, l.k.rows, l.v.rows);
        }
        if (f.has(p + "attn_q.bias")) {  // Linear bias (layers.rs:20-21,59-61)
            I.qkv_bias = 1;
            float *bq, *bk, *bv;
            CW_TRY(load_vec(m, f, p + "attn_q.bias", qd, &bq));
            CW_TRY(load_vec(m, f, p + "attn_k.bias", kvd, &bk));
            CW_TRY(load_vec(m, f, p + "attn_v.bias", kvd, &bv));
            const size_t lq = qd / T, lkv = kvd / T;  // this rank's slice of each
            void* pb;
            CW_TRY(dev_alloc(m, (lq + 2 * lkv) * 4, &pb));
            cudaStream_t st = m->ctx->stream;
            CW_CUDA(cudaMemcpyAsync(pb, bq + lq * r, lq * 4, cudaMemcpyDeviceToDevice, st));
            CW_CUDA(cudaMemcpyAsync((float*)pb + lq, bk + lkv * r, lkv * 4,
                                    cudaMemcpyDeviceToDevice, st));
            CW_CUDA(cudaMemcpyAsync((float*)pb + lq + lkv, bv + lkv * r, lkv * 4,
                                    cudaMemcpyDeviceToDevice, st));
            CW_CUDA(cudaStreamSynchronize(st));
            l.qkv_bias = (float*)pb;
        }
        CW_TRY(T > 1 ? load_q4_slice(m, f, {p + "attn_output.weight"}, qd, false, 1, 0, T, r, &l.wo)
                     : load_proj(m, f, {p + "attn_output.weight"}, qd, false, &l.wo));
        if (I.qk_norm) {
            CW_TRY(load_vec(m, f, p + "attn_q_norm.weight", I.head_dim, &l.q_norm));
            CW_TRY(load_vec(m, f, p + "attn_k_norm.weight", I.head_dim, &l.k_norm));
        }
        CW_TRY(load_vec(m, f, p + "ffn_norm.weight", I.dim, &l.ffn_norm));
        const std::vector<std::string> gu = {p + "ffn_gate.weight", p + "ffn_up.weight"};
        CW_TRY(T > 1 ? load_q4_slice(m, f, gu, I.dim, true, T, r, 1, 0, &l.gate_up)
                     : load_proj(m, f, gu, I.dim, true, &l.gate_up));
        CW_TRY(T > 1
                   ? load_q4_slice(m, f, {p + "ffn_down.weight"}, I.hidden, false, 1, 0, T, r, &l.down)
                   : load_proj(m, f, {p + "ffn_down.weight"}, I.hidden, false, &l.down));
        if (I.post_norms) {
            CW_TRY(load_vec(m, f, p + "post_attention_norm.weight", I.dim, &l.post_attn));
            CW_TRY(load_vec(m, f, p + "post_ffw_norm.weight", I.dim, &l.post_ffw));
        }
    }
    CW_TRY(load_vec(m, f, "output_norm.weight", I.dim, &m->final_norm));
    {  // Q4_0 planes, or raw k-quant rows (dequantised per element by the embed kernels)
        const GgufTensor* te = f.tensor("token_embd.weight");
        CW_CHECK(te, CW_ERR_NOT_FOUND, "missing tensor token_embd.weight");
        if (te->type != GGML_Q6_K && is_raw(te->type))
            CW_TRY(load_kq(m, f, {"token_embd.weight"}, I.dim, false, &m->embed));
        else
            CW_TRY(load_q4_or_q6k(m, f, "token_embd.weight", I.dim, &m->embed));
    }
    CW_CHECK(m->embed.rows == (int)I.vocab, CW_ERR_FORMAT, "token_embd has %d rows, vocab %u",
             m->embed.rows, I.vocab);
    if (T > 1) {  // this rank's vocabulary rows of the (untied or tied) head
        const std::string hn = f.has("output.weight") ? "output.weight" : "token_embd.weight";
        const GgufTensor* t = f.tensor(hn);
        if (t->type == GGML_Q6_K)
            CW_TRY(load_q6k(m, t, I.dim, &m->head, T, r));
        else
            CW_TRY(load_q4_slice(m, f, {hn}, I.dim, false, T, r, 1, 0, &m->head));
    } else if (f.has("output.weight")) {  // untied head; tied otherwise (qwen3.rs:93-98)
        CW_TRY(load_proj(m, f, {"output.weight"}, I.dim, false, &m->head));
    } else {
        m->head = m->embed;
    }
    CW_TRY(rope_table(m->ctx, I.head_dim, I.rope_theta, &m->inv_freq));
    m->info_full = I;
    if (T > 1) {  // the kernels see this rank's share
        I.n_heads /= T;
        I.n_kv /= T;
        I.hidden /= T;
        I.vocab /= T;
        m->vocab_offset = I.vocab * r;
        CW_CHECK(m->head.rows == (int)I.vocab, CW_ERR_FORMAT, "head shard has %d rows",
                 m->head.rows);
    }
    return CW_OK;
}

}  // namespace cw

// ===========================================================================
// session
// ===========================================================================
namespace cw {

static int sess_alloc(cw_session* s, size_t nbytes, void** p) {
    cw_buf b;
    BufEntry* e;
    CW_TRY(buf_new(s->ctx, nbytes, BUF_PERSISTENT, &b, &e));
    s->owned.push_back(b);
    CW_CUDA(cudaMemsetAsync(e->ptr, 0, nbytes, s->ctx->stream));
    *p = e->ptr;
    return CW_OK;
}

// Enqueue one generate step (decode: with lm_head + argmax).
static int enqueue_step_core(cw_session* s, bool decode);

// One step: the decode kernels, then (decode steps with sampling or stop
// tokens configured) the sampling kernel that may replace the argmax.
const Tap* find_tap(const cw_session* s, int kind, uint32_t layer) {
    for (const Tap& t : s->taps)
        if (t.kind == kind && t.layer == layer) return &t;
    return nullptr;
}

static int tap_copy(cw_session* s, int kind, uint32_t li, const float* src) {
    const Tap* t = find_tap(s, kind, li);
    if (!t) return CW_OK;
    k_tap<<<(unsigned)((t->len + 255) / 256), 256, 0, s->ctx->stream>>>(
        src, (int)t->len, t->ring, (int)t->cap, s->st);
    return check_launch("hook tap");
}

static int enqueue_step(cw_session* s, bool decode) {
    // taps read intermediates the persistent step never materialises
    const bool persistent = s->plan && s->taps.empty();
    CW_TRY(persistent ? step_enqueue(s, decode) : enqueue_step_core(s, decode));
    return decode && sample_active(s) ? sample_enqueue(s) : CW_OK;
}

static int enqueue_step_core(cw_session* s, bool decode) {
    cw_model* m = s->m;
    cw_ctx* ctx = s->ctx;
    const cw_model_info& I = m->info;
    const int qd = I.n_heads * I.head_dim;
    const bool post = I.post_norms != 0;
    // Tensor parallelism: each rank's O and down projections produce a partial
    // sum over its heads / FFN columns; it goes to tmp, is all-reduced over the
    // ranks, and is added to the residual by the next prologue, as the
    // post-norm families do with their normed branch outputs (no post norm
    // then: post_w stays null).
    const bool tp = m->tp_world > 1;
    const bool p2p = tp && p2p_on(s);  // NVLink peer all-reduces (cw_tp_p2p.cu), else NCCL
    const bool defer = post || tp;
    const int unit = I.norm_kind == 1;
    // With the context profiler on (direct launches only), every kernel is
    // bracketed by CUDA events under its stage name.
    std::unique_ptr<OpScope> sc;
    auto stage = [&](const char* name) {
        sc.reset();
        if (ctx->profiling) sc.reset(new OpScope(ctx, name));
    };
    stage("embed");
    CW_TRY(launch_k(ctx, k_embed, dim3(1), dim3(256), 0, m->embed.payload, m->embed.scales,
                    m->embed.type, (int)I.dim, I.embed_scale, (const DevState*)s->st,
                    s->hidden));
    CW_TRY(check_launch("embed"));
    for (uint32_t li = 0; li < I.n_layers; li++) {
        stage("attn_in");
        const Layer& l = m->L[li];
        FArgs a{};
        // attn_in: x = rmsnorm(h) with h = hidden, or (post-norm families,
        // li > 0) h = hidden_b + postnorm(tmp) written back to hidden.
        a.payload = l.qkv.payload;
        a.scales = l.qkv.scales;
        a.K = I.dim;
        a.N = l.qkv.rows;
        if (defer && li > 0) {
            a.base = s->hidden_b;
            a.delta = s->tmp;
            a.post_w = post ? m->L[li - 1].post_ffw : nullptr;
            a.h_out = s->hidden;
        } else {
            a.base = s->hidden;
        }
        a.norm_w = l.attn_norm;
        a.eps = I.eps;
        a.unit = unit;
        a.y = s->qkv;
        a.bias = l.qkv_bias;
        if (!l.qkv_split) {
            CW_TRY((proj<PRO_NORM, EPI_STORE>(ctx, l.qkv, a)));
        } else {  // the slices of the qkv vector by weight type (one prologue each)
            size_t off = 0;
            for (const QW* w : {&l.q, &l.k, &l.v}) {
                if (!w->rows) continue;
                FArgs b = a;
                b.y = s->qkv + off;
                b.bias = l.qkv_bias ? l.qkv_bias + off : nullptr;
                if (off) b.h_out = nullptr;  // written once
                CW_TRY((proj<PRO_NORM, EPI_STORE>(ctx, *w, b)));
                off += (size_t)w->rows;
            }
        }

        stage("attention");
        AArgs t{};
        t.qkv = s->qkv;
        t.q_norm = l.q_norm;
        t.k_norm = l.k_norm;
        t.eps = I.eps;
        t.inv_freq = m->inv_freq;
        t.kc = s->kc + (size_t)li * I.n_kv * s->max_seq * I.head_dim;
        t.vc = s->vc + (size_t)li * I.n_kv * s->max_seq * I.head_dim;
        t.max_seq = (int)s->max_seq;
        t.out = s->attn;
        t.part = s->part;
        t.counters = s->counters;
        t.n_heads = I.n_heads;
        t.n_kv = I.n_kv;
        t.hd = I.head_dim;
        t.n_splits = s->n_splits;
        t.window = (I.sliding_window && li % 2 == 0) ? (int)I.sliding_window : 0;
        t.scale = powf((float)I.head_dim, -0.5f);  // attention.rs:18
        t.softcap = I.attn_softcap;
        t.st = s->st;
        t.q_out = find_tap(s, TAP_Q, li) ? s->qtap : nullptr;
        CW_TRY(launch_fattn(ctx, t));
        CW_TRY(tap_copy(s, TAP_Q, li, s->qtap));

        stage("attn_out");
        FArgs o{};
        o.payload = l.wo.payload;
        o.scales = l.wo.scales;
        o.K = qd;
        o.N = I.dim;
        o.x = s->attn;
        o.y = defer ? s->tmp : s->hidden;
        CW_TRY(defer ? (proj<PRO_X, EPI_STORE>(ctx, l.wo, o)) : (proj<PRO_X, EPI_RESID>(ctx, l.wo, o)));
        if (tp)
            CW_TRY(p2p ? p2p_allreduce(s, s->tmp, 2 * (int)li)
                       : tp_sum_f32(m->nccl, s->tmp, I.dim, ctx->stream));
        if (!defer) CW_TRY(tap_copy(s, TAP_POST_ATTN, li, s->hidden));

        stage("ffn_in");
        FArgs f{};
        f.payload = l.gate_up.payload;
        f.scales = l.gate_up.scales;
        f.K = I.dim;
        f.N = l.gate_up.rows;
        f.base = s->hidden;
        if (defer) {
            f.delta = s->tmp;
            f.post_w = post ? l.post_attn : nullptr;
            f.h_out = s->hidden_b;
        }
        f.norm_w = l.ffn_norm;
        f.eps = I.eps;
        f.unit = unit;
        f.y = s->act;
        f.geglu = I.activation == 1;
        CW_TRY((proj<PRO_NORM, EPI_GLU>(ctx, l.gate_up, f)));
        if (post) CW_TRY(tap_copy(s, TAP_POST_ATTN, li, s->hidden_b));  // h_out of this prologue

        stage("ffn_out");
        FArgs d{};
        d.payload = l.down.payload;
        d.scales = l.down.scales;
        d.K = I.hidden;
        d.N = I.dim;
        d.x = s->act;
        d.y = defer ? s->tmp : s->hidden;
        CW_TRY(defer ? (proj<PRO_X, EPI_STORE>(ctx, l.down, d)) : (proj<PRO_X, EPI_RESID>(ctx, l.down, d)));
        if (tp)
            CW_TRY(p2p ? p2p_allreduce(s, s->tmp, 2 * (int)li + 1)
                       : tp_sum_f32(m->nccl, s->tmp, I.dim, ctx->stream));
        if (!defer) {
            CW_TRY(tap_copy(s, TAP_LAYER_OUT, li, s->hidden));
        } else if (const Tap* tp = find_tap(s, TAP_LAYER_OUT, li)) {
            // the next prologue forms hidden_b + postnorm(tmp); form it here for the tap
            k_tap_postadd<<<1, 256, 0, ctx->stream>>>(s->hidden_b, s->tmp, l.post_ffw, unit, I.eps,
                                                      (int)I.dim, tp->ring, (int)tp->cap, s->st);
            CW_TRY(check_launch("hook tap"));
        }
    }
    if (decode) {
        stage("lm_head");
        FArgs h{};
        h.payload = m->head.payload;
        h.scales = m->head.scales;
        h.K = I.dim;
        h.N = (int)I.vocab;
        h.key_offset = m->vocab_offset;
        if (defer) {
            h.base = s->hidden_b;
            h.delta = s->tmp;
            h.post_w = post ? m->L[I.n_layers - 1].post_ffw : nullptr;
        } else {
            h.base = s->hidden;
        }
        h.norm_w = m->final_norm;
        h.xn_out = s->xnorm;
        h.eps = I.eps;
        h.unit = unit;
        h.y = s->logits;
        h.softcap = I.final_softcap;
        h.key = &s->st->key;
        CW_TRY((proj<PRO_NORM, EPI_HEAD>(ctx, m->head, h)));
        // the best (logit, index) key over the vocabulary shards
        if (tp) CW_TRY(p2p ? p2p_key(s) : tp_max_u64(m->nccl, &s->st->key, 1, ctx->stream));
    }
    stage("finalize");
    CW_TRY(launch_k(ctx, k_finalize, dim3(1), dim3(1), 0, s->st, (const unsigned*)s->prompt,
                    s->toks, decode ? 1 : 0, p2p ? 2u * I.n_layers : 0u));
    sc.reset();
    return check_launch("finalize");
}

static int build_graph(cw_session* s, bool decode, cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    CW_CUDA(cudaStreamBeginCapture(s->ctx->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(s, decode);
    cudaError_t e = cudaStreamEndCapture(s->ctx->stream, &g);
    if (rc != CW_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (e != cudaSuccess) return set_error(CW_ERR_CUDA, "graph capture: %s", cudaGetErrorString(e));
    e = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess)
        return set_error(CW_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(e));
    return CW_OK;
}

static void destroy_graphs(cw_session* s) {
    for (auto& row : s->graphs)
        for (auto& g : row)
            if (g) {
                cudaGraphExecDestroy(g);
                g = nullptr;
            }
}

bool model_q4_only(const cw_model* m, bool head) {
    if (head && m->head.type != GGML_Q4_0) return false;
    for (const Layer& l : m->L)
        if (l.qkv_split || l.qkv.type != GGML_Q4_0 || l.wo.type != GGML_Q4_0 ||
            l.gate_up.type != GGML_Q4_0 || l.down.type != GGML_Q4_0)
            return false;
    return true;
}

// Host counters from the device state (EOS may have ended the sequence
// inside a run of steps).
int sync_counts(cw_session* s) {
    DevState h;
    CW_CUDA(cudaMemcpyAsync(&h, s->st, sizeof h, cudaMemcpyDeviceToHost, s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    s->n_produced = (size_t)h.n_produced;
    s->stopped = h.stopped != 0;
    return CW_OK;
}

static int run_step(cw_session* s) {
    bool decode = !(s->host_pos + 1 < s->n_prompt);
    CW_CHECK(s->host_pos < s->max_seq, CW_ERR_INVALID_ARG,
             "session is full: position %zu, max_seq %zu", s->host_pos, s->max_seq);
    if (s->use_graph) {
        cudaGraphExec_t* g = &s->graphs[step_variant(s)][decode ? 1 : 0];
        if (!*g) CW_TRY(build_graph(s, decode, g));
        CW_CUDA(cudaGraphLaunch(*g, s->ctx->stream));
    } else {
        CW_TRY(enqueue_step(s, decode));
    }
    s->host_pos++;
    if (decode) s->n_produced++;
    return CW_OK;
}

}  // namespace cw

using namespace cw;

extern "C" {

int cw_model_load_gguf(cw_ctx* ctx, const char* path, cw_model** out) {
    clear_error();
    CW_CHECK(ctx && path && out, CW_ERR_INVALID_ARG, "cw_model_load_gguf: bad arguments");
    cudaSetDevice(ctx->device);
    cw_model* m = new cw_model();
    m->ctx = ctx;
    int rc = model_load(m, path);
    if (rc != CW_OK) {
        std::string msg = cw_last_error();
        cw_model_free(m);
        return set_error(rc, "%s", msg.c_str());
    }
    *out = m;
    return CW_OK;
}

int cw_tp_unique_id(uint8_t* id, size_t n) {
    clear_error();
    CW_CHECK(id && n >= CW_TP_ID_BYTES, CW_ERR_INVALID_ARG,
             "cw_tp_unique_id: need a buffer of %d bytes", CW_TP_ID_BYTES);
    memset(id, 0, n);
    return tp_unique_id(id, n);
}

int cw_model_load_gguf_tp(cw_ctx* ctx, const char* path, int rank, int world, const uint8_t* id,
                          cw_model** out) {
    clear_error();
    CW_CHECK(ctx && path && out && id && world >= 1 && world <= 64 && rank >= 0 && rank < world,
             CW_ERR_INVALID_ARG, "cw_model_load_gguf_tp: bad arguments");
    if (world == 1) return cw_model_load_gguf(ctx, path, out);
    cudaSetDevice(ctx->device);
    cw_model* m = new cw_model();
    m->ctx = ctx;
    m->tp_rank = rank;
    m->tp_world = world;
    // the communicator first: the ranks read the same file, so a load error
    // comes on every rank, after all of them have joined
    int rc = tp_comm_init(id, rank, world, &m->nccl);
    if (rc == CW_OK) rc = model_load(m, path);
    if (rc != CW_OK) {
        std::string msg = cw_last_error();
        cw_model_free(m);
        return set_error(rc, "%s", msg.c_str());
    }
    *out = m;
    return CW_OK;
}

int cw_model_tp_info(cw_model* m, int* rank, int* world, uint32_t* vocab_offset,
                     uint32_t* vocab_local) {
    clear_error();
    CW_CHECK(m, CW_ERR_INVALID_ARG, "cw_model_tp_info: model is NULL");
    if (rank) *rank = m->tp_rank;
    if (world) *world = m->tp_world;
    if (vocab_offset) *vocab_offset = m->vocab_offset;
    if (vocab_local) *vocab_local = m->info.vocab;
    return CW_OK;
}

int cw_model_free(cw_model* m) {
    if (!m) return CW_OK;
    cudaSetDevice(m->ctx->device);
    cudaStreamSynchronize(m->ctx->stream);
    tp_comm_destroy(m->nccl);
    m->nccl = nullptr;
    for (cw_buf b : m->owned) {
        auto it = m->ctx->bufs.find(b);
        if (it != m->ctx->bufs.end()) {
            cudaFree(it->second.ptr);
            m->ctx->bufs.erase(it);
        }
    }
    for (void* p : m->packed) cudaFree(p);
    for (void* p : m->grp_tiles) cudaFree(p);
    delete m;
    return CW_OK;
}

int cw_model_get_info(cw_model* m, cw_model_info* info) {
    clear_error();
    CW_CHECK(m && info, CW_ERR_INVALID_ARG, "cw_model_get_info: bad arguments");
    if (m->tp_world > 1) {  // the whole model's shapes; weight bytes held by this rank
        *info = m->info_full;
        info->weight_bytes = m->info.weight_bytes;
    } else {
        *info = m->info;
    }
    return CW_OK;
}

int cw_session_create(cw_model* m, size_t max_seq, cw_session** out) {
    clear_error();
    CW_CHECK(m && out && max_seq > 0 && max_seq < (1u << 24), CW_ERR_INVALID_ARG,
             "cw_session_create: bad arguments");
    cw_ctx* ctx = m->ctx;
    cudaSetDevice(ctx->device);
    const cw_model_info& I = m->info;
    cw_session* s = new cw_session();
    s->m = m;
    s->ctx = ctx;
    s->max_seq = max_seq;
    int rc = CW_OK;
    auto A = [&](size_t n, void** p) {
        if (rc == CW_OK) rc = sess_alloc(s, n, p);
    };
    size_t kv = (size_t)I.n_layers * I.n_kv * max_seq * I.head_dim * 4;
    size_t qd = (size_t)I.n_heads * I.head_dim, kvd = (size_t)I.n_kv * I.head_dim;
    A(kv, (void**)&s->kc);
    A(kv, (void**)&s->vc);
    A(I.dim * 4, (void**)&s->hidden);
    A(I.dim * 4, (void**)&s->hidden_b);
    A(I.dim * 4, (void**)&s->tmp);
    A((qd + 2 * kvd) * 4, (void**)&s->qkv);
    A(qd * 4, (void**)&s->attn);
    A((size_t)I.hidden * 4, (void**)&s->act);
    A((size_t)I.vocab * 4, (void**)&s->logits);
    A(I.dim * 4, (void**)&s->xnorm);
    // split-KV: about two CTAs per SM, at most one split per 8 keys
    s->n_splits = std::max(1, std::min<int>((int)((max_seq + 7) / 8),
                                            2 * ctx->sm_count / (int)I.n_kv));
    // split rows of (head_dim + 4) floats: the persistent step's 16-byte-aligned layout
    A((size_t)I.n_heads * s->n_splits * (I.head_dim + 4) * 4, (void**)&s->part);
    A(max_seq * 4, (void**)&s->prompt);
    A(max_seq * 4, (void**)&s->toks);
    A((size_t)I.n_kv * 4, (void**)&s->counters);
    A(sizeof(DevState), (void**)&s->st);
    A(2 * sizeof(unsigned long long), (void**)&s->bar);
    // fixed-point residual accumulators of the persistent step (O-projection
    // and FFN partial sums by layer parity)
    A((size_t)4 * I.dim * sizeof(long long), (void**)&s->racc);
    A((size_t)2 * I.dim * sizeof(float), (void**)&s->hid2);
    A((size_t)2 * I.n_layers * I.n_kv * sizeof(unsigned), (void**)&s->rdy);
    A((size_t)sample_params_size(), &s->smp_dev);
    A(qd * 4, (void**)&s->qtap);
    A((qd + 2 * kvd) * 8, (void**)&s->qkv_words);
    if (rc == CW_OK) rc = sample_params_write(s);
    if (rc == CW_OK && (cudaMallocHost(&s->h_tok, sizeof(unsigned)) != cudaSuccess ||
                        cudaMallocHost(&s->h_tok_in, sizeof(unsigned)) != cudaSuccess))
        rc = set_error(CW_ERR_OOM, "pinned host allocation failed");
    if (rc == CW_OK && cudaStreamSynchronize(ctx->stream) != cudaSuccess)
        rc = set_error(CW_ERR_CUDA, "session setup failed");
    if (rc == CW_OK && s->use_persistent && step_default(m, s)) rc = step_plan_create(s);
    if (rc != CW_OK) {
        std::string msg = cw_last_error();
        cw_session_free(s);
        return set_error(rc, "%s", msg.c_str());
    }
    *out = s;
    return CW_OK;
}

int cw_session_free(cw_session* s) {
    if (!s) return CW_OK;
    cudaSetDevice(s->ctx->device);
    cudaStreamSynchronize(s->ctx->stream);
    destroy_graphs(s);
    step_plan_free(s);
    p2p_free(s);
    for (cw_buf b : s->owned) {
        auto it = s->ctx->bufs.find(b);
        if (it != s->ctx->bufs.end()) {
            cudaFree(it->second.ptr);
            s->ctx->bufs.erase(it);
        }
    }
    if (s->h_tok) cudaFreeHost(s->h_tok);
    if (s->h_tok_in) cudaFreeHost(s->h_tok_in);
    if (s->pf_mem) cudaFree(s->pf_mem);
    delete s;
    return CW_OK;
}

int cw_session_set_graph(cw_session* s, int use_graph) {
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_set_graph: session is NULL");
    s->use_graph = use_graph != 0;
    return CW_OK;
}

int cw_session_set_persistent(cw_session* s, int on) {
    clear_error();
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_set_persistent: session is NULL");
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    // captured graphs hold one path or the other
    destroy_graphs(s);
    CW_CHECK(on >= 0 && on <= 2, CW_ERR_INVALID_ARG, "cw_session_set_persistent: mode %d", on);
    s->use_persistent = on != 0;
    if (!on) {
        step_plan_free(s);
        return CW_OK;
    }
    if (!s->plan) {
        CW_CHECK(step_supported(s->m, s), CW_ERR_UNSUPPORTED,
                 "the persistent step does not cover this model family");
        CW_TRY(step_plan_create(s));
    }
    return CW_OK;
}

int cw_session_tp_handle(cw_session* s, uint8_t* out, size_t n) {
    clear_error();
    CW_CHECK(s && out && n >= CW_TP_HANDLE_BYTES, CW_ERR_INVALID_ARG,
             "cw_session_tp_handle: bad arguments");
    cudaSetDevice(s->ctx->device);
    return p2p_handle(s, out);
}

int cw_session_tp_attach(cw_session* s, const uint8_t* handles, size_t n) {
    clear_error();
    CW_CHECK(s && handles, CW_ERR_INVALID_ARG, "cw_session_tp_attach: bad arguments");
    CW_CHECK(n >= (size_t)s->m->tp_world * CW_TP_HANDLE_BYTES, CW_ERR_INVALID_ARG,
             "cw_session_tp_attach: %zu bytes for %d ranks", n, s->m->tp_world);
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    destroy_graphs(s);  // captured steps hold the NCCL all-reduces
    return p2p_attach(s, handles);
}

int cw_session_inject_stall(cw_session* s, uint32_t wait_us) {
    clear_error();
    CW_CHECK(s && wait_us > 0, CW_ERR_INVALID_ARG, "cw_session_inject_stall: bad arguments");
    CW_CHECK(s->use_persistent && s->plan, CW_ERR_UNSUPPORTED,
             "cw_session_inject_stall: the session is not on the persistent step");
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaMemcpyAsync(&s->st->stall_us, &wait_us, sizeof(uint32_t), cudaMemcpyHostToDevice,
                            s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    return CW_OK;
}

int cw_session_persistent(cw_session* s, int* on) {
    CW_CHECK(s && on, CW_ERR_INVALID_ARG, "cw_session_persistent: bad arguments");
    *on = s->plan != nullptr;
    return CW_OK;
}

int cw_session_begin(cw_session* s, const uint32_t* prompt, size_t n_prompt) {
    clear_error();
    CW_CHECK(s && prompt && n_prompt > 0, CW_ERR_INVALID_ARG,
             "cw_session_begin: the prompt must hold at least one token");
    CW_CHECK(n_prompt <= s->max_seq, CW_ERR_INVALID_ARG, "prompt of %zu tokens exceeds max_seq %zu",
             n_prompt, s->max_seq);
    for (size_t i = 0; i < n_prompt; i++)
        CW_CHECK(prompt[i] < s->m->vocab_full, CW_ERR_INVALID_ARG,
                 "prompt token %u at %zu is outside the vocabulary (%u)", prompt[i], i,
                 s->m->vocab_full);
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaMemcpyAsync(s->prompt, prompt, n_prompt * 4, cudaMemcpyHostToDevice, s->ctx->stream));
    k_begin<<<1, 1, 0, s->ctx->stream>>>(s->st, s->prompt, (int)n_prompt, s->bar);
    CW_TRY(check_launch("session begin"));
    // the persistent step's accumulators start from zero (a step that timed
    // out may have left partial sums behind)
    CW_CUDA(cudaMemsetAsync(s->racc, 0, (size_t)4 * s->m->info.dim * sizeof(long long),
                            s->ctx->stream));
    CW_CUDA(cudaMemsetAsync(s->rdy, 0,
                            (size_t)2 * s->m->info.n_layers * s->m->info.n_kv * sizeof(unsigned),
                            s->ctx->stream));
    {  // tag 0, which no step uses
        const cw_model_info& I = s->m->info;
        CW_CUDA(cudaMemsetAsync(s->qkv_words, 0, (size_t)(I.n_heads + 2 * I.n_kv) * I.head_dim * 8,
                                s->ctx->stream));
    }
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    s->host_pos = 0;
    s->n_prompt = n_prompt;
    s->n_produced = 0;
    s->stopped = false;
    return CW_OK;
}


int cw_session_set_sampling(cw_session* s, float temperature, uint32_t top_k, float top_p,
                            uint64_t seed) {
    clear_error();
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_set_sampling: session is NULL");
    CW_CHECK(temperature == temperature && top_p >= 0.f && top_p <= 1.f, CW_ERR_INVALID_ARG,
             "cw_session_set_sampling: temperature must be a number and top_p in [0, 1]");
    CW_CHECK(!(temperature > 0.f) || s->m->tp_world == 1, CW_ERR_UNSUPPORTED,
             "cw_session_set_sampling: a tensor-parallel model decodes greedily (each rank "
             "holds a slice of the logits)");
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    destroy_graphs(s);  // the decode graph holds the sampling launch or not
    s->smp_temperature = temperature > 0.f ? temperature : 0.f;
    s->smp_top_k = top_k;
    s->smp_top_p = top_p;
    s->smp_seed = seed;
    return sample_params_write(s);
}

int cw_session_set_eos(cw_session* s, const uint32_t* ids, size_t n) {
    clear_error();
    CW_CHECK(s && (ids || n == 0) && n <= CW_MAX_EOS, CW_ERR_INVALID_ARG,
             "cw_session_set_eos: at most %d stop tokens", CW_MAX_EOS);
    for (size_t i = 0; i < n; i++)
        CW_CHECK(ids[i] < s->m->vocab_full, CW_ERR_INVALID_ARG,
                 "cw_session_set_eos: token %u outside the vocabulary", ids[i]);
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    destroy_graphs(s);
    s->eos.assign(ids, ids + n);
    return sample_params_write(s);
}

static int tap_kind(const char* name) {
    if (!name) return -1;
    if (!strcmp(name, "q")) return TAP_Q;
    if (!strcmp(name, "post_attn")) return TAP_POST_ATTN;
    if (!strcmp(name, "layer_out")) return TAP_LAYER_OUT;
    return -1;
}

int cw_session_add_tap(cw_session* s, const char* name, uint32_t layer, size_t cap) {
    clear_error();
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_add_tap: session is NULL");
    const int kind = tap_kind(name);
    CW_CHECK(kind >= 0, CW_ERR_INVALID_ARG,
             "cw_session_add_tap: unknown tap '%s' (q, post_attn, layer_out)", name ? name : "");
    CW_CHECK(s->m->tp_world == 1, CW_ERR_UNSUPPORTED,
             "cw_session_add_tap: taps are not available on a tensor-parallel model");
    const cw_model_info& I = s->m->info;
    CW_CHECK(layer < I.n_layers && cap > 0 && cap <= s->max_seq, CW_ERR_INVALID_ARG,
             "cw_session_add_tap: layer %u of %u, cap %zu (1..max_seq)", layer, I.n_layers, cap);
    CW_CHECK(!find_tap(s, kind, layer), CW_ERR_INVALID_ARG, "tap %s/%u already added", name, layer);
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    destroy_graphs(s);  // the captured step gains the tap's copy
    Tap t;
    t.kind = kind;
    t.layer = layer;
    t.cap = cap;
    t.len = kind == TAP_Q ? (size_t)I.n_heads * I.head_dim : I.dim;
    CW_TRY(sess_alloc(s, t.cap * t.len * 4, (void**)&t.ring));
    t.buf = s->owned.back();
    CW_CUDA(cudaMemsetAsync(t.ring, 0, t.cap * t.len * 4, s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    s->taps.push_back(t);
    return CW_OK;
}

int cw_session_clear_taps(cw_session* s) {
    clear_error();
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_clear_taps: session is NULL");
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    destroy_graphs(s);
    for (const Tap& t : s->taps) {
        auto it = s->ctx->bufs.find(t.buf);
        if (it != s->ctx->bufs.end()) {
            cudaFree(it->second.ptr);
            s->ctx->bufs.erase(it);
        }
        s->owned.erase(std::remove(s->owned.begin(), s->owned.end(), t.buf), s->owned.end());
    }
    s->taps.clear();
    return CW_OK;
}

int cw_session_read_tap(cw_session* s, const char* name, uint32_t layer, size_t pos, float* out,
                        size_t len) {
    clear_error();
    CW_CHECK(s && out, CW_ERR_INVALID_ARG, "cw_session_read_tap: bad arguments");
    const Tap* t = find_tap(s, tap_kind(name), layer);
    CW_CHECK(t, CW_ERR_INVALID_ARG, "cw_session_read_tap: no tap %s/%u", name ? name : "", layer);
    CW_CHECK(len == t->len, CW_ERR_INVALID_ARG, "cw_session_read_tap: the tap holds %zu floats",
             t->len);
    CW_CHECK(pos < s->host_pos && pos + t->cap >= s->host_pos, CW_ERR_INVALID_ARG,
             "cw_session_read_tap: position %zu is not among the last %zu recorded (next %zu)",
             pos, t->cap, s->host_pos);
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaMemcpyAsync(out, t->ring + (pos % t->cap) * t->len, t->len * 4,
                            cudaMemcpyDeviceToHost, s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    return check_device_status(s->ctx);
}

int cw_session_stopped(cw_session* s, int* stopped) {
    clear_error();
    CW_CHECK(s && stopped, CW_ERR_INVALID_ARG, "cw_session_stopped: bad arguments");
    cudaSetDevice(s->ctx->device);
    CW_TRY(sync_counts(s));
    *stopped = s->stopped ? 1 : 0;
    return CW_OK;
}

int cw_session_prefill(cw_session* s, size_t* n_done) {
    clear_error();
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_prefill: session is NULL");
    CW_CHECK(s->n_prompt > 0, CW_ERR_INVALID_ARG, "cw_session_prefill: call cw_session_begin first");
    CW_CHECK(s->m->tp_world == 1, CW_ERR_UNSUPPORTED,
             "cw_session_prefill: not available on a tensor-parallel model (the prompt runs "
             "through cw_session_run)");
    CW_CHECK(model_q4_only(s->m, false), CW_ERR_UNSUPPORTED,
             "cw_session_prefill: the tensor-core prefill takes Q4_0 projections (the prompt "
             "runs through cw_session_run)");
    cudaSetDevice(s->ctx->device);
    CW_TRY(session_prefill(s, n_done));
    return check_launch("session prefill");
}

int cw_session_set_prefill_chunk(cw_session* s, size_t rows) {
    clear_error();
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_set_prefill_chunk: session is NULL");
    CW_CHECK(rows <= 4096, CW_ERR_INVALID_ARG,
             "cw_session_set_prefill_chunk: %zu rows (1..4096, or 0 for the default)", rows);
    s->pf_chunk = rows;
    return CW_OK;
}

int cw_session_read_kv(cw_session* s, uint32_t layer, size_t n_pos, float* k, float* v) {
    clear_error();
    CW_CHECK(s && k && v && layer < s->m->info.n_layers && n_pos <= s->max_seq,
             CW_ERR_INVALID_ARG, "cw_session_read_kv: bad arguments");
    cudaSetDevice(s->ctx->device);
    const cw_model_info& I = s->m->info;
    const size_t row = (size_t)I.head_dim * 4, per_head = s->max_seq * I.head_dim;
    const size_t base = (size_t)layer * I.n_kv * per_head;
    for (uint32_t g = 0; g < I.n_kv; g++) {
        CW_CUDA(cudaMemcpyAsync(k + (size_t)g * n_pos * I.head_dim, s->kc + base + g * per_head,
                                n_pos * row, cudaMemcpyDeviceToHost, s->ctx->stream));
        CW_CUDA(cudaMemcpyAsync(v + (size_t)g * n_pos * I.head_dim, s->vc + base + g * per_head,
                                n_pos * row, cudaMemcpyDeviceToHost, s->ctx->stream));
    }
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    return check_device_status(s->ctx);
}

int cw_session_run(cw_session* s, size_t n_steps, size_t* n_produced) {
    clear_error();
    CW_CHECK(s, CW_ERR_INVALID_ARG, "cw_session_run: session is NULL");
    CW_CHECK(s->n_prompt > 0, CW_ERR_INVALID_ARG, "cw_session_run: call cw_session_begin first");
    cudaSetDevice(s->ctx->device);
    size_t before = s->n_produced;
    for (size_t i = 0; i < n_steps; i++) CW_TRY(run_step(s));
    if (!s->eos.empty()) CW_TRY(sync_counts(s));  // an EOS may have stopped the run
    if (n_produced) *n_produced = s->n_produced - before;
    return check_launch("session run");
}

int cw_session_tokens(cw_session* s, uint32_t* out, size_t cap, size_t* n) {
    clear_error();
    CW_CHECK(s && n, CW_ERR_INVALID_ARG, "cw_session_tokens: bad arguments");
    cudaSetDevice(s->ctx->device);
    CW_TRY(sync_counts(s));
    size_t k = std::min(cap, s->n_produced);
    if (k && out)
        CW_CUDA(cudaMemcpyAsync(out, s->toks, k * 4, cudaMemcpyDeviceToHost, s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    *n = s->n_produced;
    return check_device_status(s->ctx);
}

int cw_session_logits(cw_session* s, float* out, size_t vocab) {
    clear_error();
    CW_CHECK(s && out && vocab == s->m->info.vocab, CW_ERR_INVALID_ARG,
             "cw_session_logits: bad arguments (vocab is %u)", s ? s->m->info.vocab : 0);
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaMemcpyAsync(out, s->logits, vocab * 4, cudaMemcpyDeviceToHost, s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    return CW_OK;
}

int cw_session_hidden(cw_session* s, float* out, size_t dim) {
    clear_error();
    CW_CHECK(s && out && dim == s->m->info.dim, CW_ERR_INVALID_ARG,
             "cw_session_hidden: bad arguments");
    cudaSetDevice(s->ctx->device);
    CW_CUDA(cudaMemcpyAsync(out, s->xnorm, dim * 4, cudaMemcpyDeviceToHost, s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    return CW_OK;
}

int cw_session_pos(cw_session* s, size_t* pos) {
    CW_CHECK(s && pos, CW_ERR_INVALID_ARG, "cw_session_pos: bad arguments");
    *pos = s->host_pos;
    return CW_OK;
}

int cw_session_step(cw_session* s, uint32_t token_in, uint32_t* token_out) {
    clear_error();
    CW_CHECK(s && token_out, CW_ERR_INVALID_ARG, "cw_session_step: bad arguments");
    CW_CHECK(s->n_prompt > 0, CW_ERR_INVALID_ARG, "cw_session_step: call cw_session_begin first");
    CW_CHECK(token_in == CW_TOKEN_DEVICE || token_in < s->m->vocab_full, CW_ERR_INVALID_ARG,
             "cw_session_step: token %u outside the vocabulary", token_in);
    cudaSetDevice(s->ctx->device);
    if (s->stopped) {  // an EOS token ended the sequence: nothing more to produce
        *token_out = CW_TOKEN_DEVICE;
        return CW_OK;
    }
    if (token_in != CW_TOKEN_DEVICE) {
        *s->h_tok_in = token_in;
        CW_CUDA(cudaMemcpyAsync(&s->st->token, s->h_tok_in, 4, cudaMemcpyHostToDevice,
                                s->ctx->stream));
    }
    bool decode = !(s->host_pos + 1 < s->n_prompt);
    size_t slot = s->n_produced;
    CW_TRY(run_step(s));
    if (decode) {
        CW_CUDA(cudaMemcpyAsync(s->h_tok, s->toks + slot, 4, cudaMemcpyDeviceToHost,
                                s->ctx->stream));
        CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
        *token_out = *s->h_tok;
        // an EOS token is returned but not counted (wasm.rs:99-101)
        if (std::find(s->eos.begin(), s->eos.end(), *token_out) != s->eos.end()) {
            s->stopped = true;
            s->n_produced--;
        }
    } else {
        CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
        *token_out = 0xffffffffu;
    }
    return CW_OK;
}

int cw_session_run_timed(cw_session* s, size_t n_steps, double* ms) {
    clear_error();
    CW_CHECK(s && ms, CW_ERR_INVALID_ARG, "cw_session_run_timed: bad arguments");
    CW_CHECK(s->n_prompt > 0, CW_ERR_INVALID_ARG, "cw_session_run_timed: call cw_session_begin first");
    cudaSetDevice(s->ctx->device);
    // build graphs outside the timed region
    if (s->use_graph) {
        cudaGraphExec_t* gp = &s->graphs[step_variant(s)][0];
        cudaGraphExec_t* gd = &s->graphs[step_variant(s)][1];
        if (!*gp && s->host_pos + 1 < s->n_prompt) CW_TRY(build_graph(s, false, gp));
        if (!*gd) CW_TRY(build_graph(s, true, gd));
    }
    cudaEvent_t e0, e1;
    CW_CUDA(cudaEventCreate(&e0));
    CW_CUDA(cudaEventCreate(&e1));
    CW_CUDA(cudaEventRecord(e0, s->ctx->stream));
    int rc = CW_OK;
    for (size_t i = 0; i < n_steps && rc == CW_OK; i++) rc = run_step(s);
    cudaEventRecord(e1, s->ctx->stream);
    cudaEventSynchronize(e1);
    float f = 0.f;
    cudaEventElapsedTime(&f, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    CW_TRY(rc);
    *ms = f;
    return check_device_status(s->ctx);
}

int cw_session_launches(cw_session* s, size_t* prompt_step, size_t* decode_step) {
    CW_CHECK(s && prompt_step && decode_step, CW_ERR_INVALID_ARG, "cw_session_launches: bad arguments");
    if (s->plan && s->taps.empty()) {  // the whole step is one persistent launch (+ sampling)
        *prompt_step = 1;
        *decode_step = 1 + (sample_active(s) ? 1 : 0);
        return CW_OK;
    }
    // embed + 5 per layer + finalize (+ lm_head/argmax on decode steps)
    size_t per = 2 + 5 * (size_t)s->m->info.n_layers;
    *prompt_step = per;
    per += s->taps.size();
    *prompt_step = per;
    *decode_step = per + 1 + (sample_active(s) ? 1 : 0);
    return CW_OK;
}

static int profile_rows(const std::map<std::string, std::pair<uint32_t, double>>& agg,
                        cw_profile_row* rows, size_t cap, size_t* n_rows) {
    std::vector<std::pair<std::string, std::pair<uint32_t, double>>> v(agg.begin(), agg.end());
    std::sort(v.begin(), v.end(),
              [](const auto& a, const auto& b) { return a.second.second > b.second.second; });
    *n_rows = v.size();
    for (size_t i = 0; i < v.size() && i < cap && rows; i++) {
        snprintf(rows[i].kernel, sizeof rows[i].kernel, "%s", v[i].first.c_str());
        rows[i].passes = v[i].second.first;
        rows[i].total_ms = v[i].second.second;
    }
    return CW_OK;
}

int cw_session_profile(cw_session* s, size_t n_steps, cw_profile_row* rows, size_t cap,
                       size_t* n_rows) {
    clear_error();
    CW_CHECK(s && n_rows, CW_ERR_INVALID_ARG, "cw_session_profile: bad arguments");
    CW_CHECK(s->n_prompt > 0, CW_ERR_INVALID_ARG, "cw_session_profile: call cw_session_begin first");
    CW_CHECK(s->host_pos + 1 >= s->n_prompt, CW_ERR_INVALID_ARG,
             "cw_session_profile: run the prompt positions first");
    cw_ctx* ctx = s->ctx;
    cudaSetDevice(ctx->device);
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    std::map<std::string, std::pair<uint32_t, double>> agg;
    if (s->plan) {  // persistent step: stage spans from in-kernel timestamps
        CW_TRY(step_profile(s, n_steps, &agg));
        return profile_rows(agg, rows, cap, n_rows);
    }
    // capture one decode step with an event pair around each kernel
    const bool pdl = ctx->pdl, prof = ctx->profiling;
    std::vector<ProfRec> saved;
    saved.swap(ctx->prof);
    ctx->pdl = false;
    ctx->profiling = true;
    cudaGraph_t g = nullptr;
    cudaGraphExec_t exec = nullptr;
    int rc = CW_OK;
    cudaError_t ce = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
    if (ce == cudaSuccess) {
        rc = enqueue_step(s, true);
        ce = cudaStreamEndCapture(ctx->stream, &g);
    }
    std::vector<ProfRec> recs;
    recs.swap(ctx->prof);
    ctx->prof.swap(saved);
    ctx->pdl = pdl;
    ctx->profiling = prof;
    if (rc == CW_OK && ce == cudaSuccess) ce = cudaGraphInstantiate(&exec, g, 0);
    if (g) cudaGraphDestroy(g);
    auto release = [&]() {
        if (exec) cudaGraphExecDestroy(exec);
        for (auto& p : recs) {
            ctx->event_pool.push_back(p.start);
            ctx->event_pool.push_back(p.stop);
        }
    };
    if (rc != CW_OK || ce != cudaSuccess) {
        release();
        if (rc != CW_OK) return rc;
        return set_error(CW_ERR_CUDA, "profile graph: %s", cudaGetErrorString(ce));
    }
    for (size_t it = 0; it < n_steps; it++) {
        if (s->host_pos >= s->max_seq) {
            release();
            return set_error(CW_ERR_INVALID_ARG, "session is full: position %zu", s->host_pos);
        }
        ce = cudaGraphLaunch(exec, ctx->stream);
        if (ce == cudaSuccess) ce = cudaStreamSynchronize(ctx->stream);
        if (ce != cudaSuccess) {
            release();
            return set_error(CW_ERR_CUDA, "profile step: %s", cudaGetErrorString(ce));
        }
        s->host_pos++;
        s->n_produced++;
        for (auto& p : recs) {
            float ms = 0.f;
            cudaEventElapsedTime(&ms, p.start, p.stop);
            auto& a = agg[p.name];
            a.first += 1;
            a.second += ms;
        }
    }
    release();
    CW_TRY(profile_rows(agg, rows, cap, n_rows));
    return check_device_status(ctx);
}

int cw_generate(cw_model* m, const uint32_t* prompt, size_t n_prompt, size_t max_new,
                uint32_t* out_tokens) {
    clear_error();
    CW_CHECK(m && prompt && out_tokens && n_prompt > 0, CW_ERR_INVALID_ARG,
             "cw_generate: bad arguments (the prompt must hold at least one token)");
    size_t want = std::max<size_t>(max_new, 1);
    cw_session* s = nullptr;
    CW_TRY(cw_session_create(m, n_prompt + want, &s));
    std::unique_ptr<cw_session, int (*)(cw_session*)> guard(s, cw_session_free);
    CW_TRY(cw_session_begin(s, prompt, n_prompt));
    size_t produced = 0;
    while (produced < want) {
        bool decode = !(s->host_pos + 1 < s->n_prompt);
        CW_TRY(run_step(s));
        if (decode) {
            // mod.rs:103: the produced token is read back every step
            CW_CUDA(cudaMemcpyAsync(s->h_tok, s->toks + produced, 4, cudaMemcpyDeviceToHost,
                                    s->ctx->stream));
            CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
            out_tokens[produced++] = *s->h_tok;
        }
    }
    return check_device_status(s->ctx);
}

}  // extern "C"
