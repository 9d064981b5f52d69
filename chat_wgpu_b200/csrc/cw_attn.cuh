// cw_attn.cuh -- split-KV single-query attention core shared by the
// stand-alone op (cw_attention) and the fused decode kernel.
//
// Semantics follow chat-wgpu src/kernels/attention.wgsl:23-96: scores
// s = scale * (q . k_j), an online softmax (running max m, denominator l,
// rescaled accumulator), GQA head h -> kv head h / (n_heads / n_kv).
// Work split: one CTA per (key range, kv head); the CTA's 4 warps take
// groups of 4 consecutive keys (warp w: keys lo + 4w .. lo + 4w + 3, then
// +16, ...), issue all 8 K/V row loads of a group before using any, and keep
// one online-softmax state per query head of the GQA group, so K/V rows are
// read once per group.  Lane l holds head dims l, l+32, ..., so a key row is
// one coalesced 128-byte read per 32 dims.
#pragma once

#include "cw_device.cuh"

namespace cw {

constexpr float REF_NEG_INF = -3.402823e38f;  // attention.wgsl:27
constexpr int ATTN_MIN_KEYS = 32;             // keys per split before splitting further
constexpr int ATTN_U = 4;                     // keys per warp iteration

// Shared memory floats needed by attn_core + attn_finish for G heads of dim
// hd, up to n_splits splits and NW warps.
__host__ __device__ constexpr size_t attn_smem_floats(int G, int hd, int n_splits, int NW = 4) {
    return (size_t)(NW + 1) * G * (hd + 2) + (size_t)G * NW + (size_t)G * (n_splits + 1);
}

// K/V load paths: read-only cache (rows written by earlier launches), plain,
// or L2-only (rows written by other CTAs of the same persistent kernel).
enum { KV_NC = 0, KV_PLAIN = 1, KV_CG = 2 };

// Splits that hold keys for a (windowed) span: at most n_splits, at least
// min_keys keys each.
__host__ __device__ __forceinline__ int attn_active_splits(int span, int n_splits,
                                                          int min_keys = ATTN_MIN_KEYS) {
    int by_len = (span + min_keys - 1) / min_keys;
    by_len = by_len < 1 ? 1 : by_len;
    return by_len < n_splits ? by_len : n_splits;
}

// Key range of split `split` of n_active over the prefix [j0, seq), with
// j0 = seq - window for a sliding-window layer.
__device__ __forceinline__ void attn_range(int seq, int window, int split, int n_active, int* jlo,
                                           int* jhi) {
    int j0 = (window > 0 && seq > window) ? seq - window : 0;
    int span = seq - j0;
    int per = (span + n_active - 1) / n_active;
    *jlo = min(seq, j0 + split * per);
    *jhi = min(seq, *jlo + per);
}

__device__ __forceinline__ int attn_span(int seq, int window) {
    return (window > 0 && seq > window) ? window : seq;
}

// Computes, for the G query heads in qg[G][hd] (global or shared memory),
// the un-normalised attention state over keys [jlo, jhi) of one kv head
// (rows kb + j*rs, vb + j*rs).  On return res[gi*(hd+2) + d] holds the
// accumulator A, res[.. + hd] the max M, res[.. + hd + 1] the denominator L.
// All NW warps call it; it ends with a barrier over them (attn_sync).
// LD selects the K/V load path (KV_NC must not be used for rows the calling
// kernel wrote).  NW warps (the CTA has NW*32 threads) take groups of four
// keys in turn.
// CTA barrier of attn_core: __syncthreads, or (NAMED) named barrier 1 over
// the NW warps that run it, for kernels with other warps that do not.
template <bool NAMED, int NW>
__device__ __forceinline__ void attn_sync() {
    if constexpr (NAMED)
        asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");
    else
        __syncthreads();
}

// U keys per warp iteration (ATTN_U; fewer where EPL is large, to bound the
// registers the iteration's K/V rows take).
template <int EPL, int GMAX, int LD = KV_NC, int NW = 4, bool NAMED = false, int U = ATTN_U>
__device__ __forceinline__ void attn_core(const float* qg, int G, int hd,
                                          const float* __restrict__ kb,
                                          const float* __restrict__ vb, long rs, int jlo, int jhi,
                                          float scale, float softcap, float* sm, float* res) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int W = hd + 2;
    float qr[GMAX][EPL], acc[GMAX][EPL], m[GMAX], l[GMAX];
#pragma unroll
    for (int gi = 0; gi < GMAX; gi++) {
        m[gi] = REF_NEG_INF;
        l[gi] = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            int d = lane + 32 * e;
            qr[gi][e] = (gi < G && d < hd) ? qg[gi * hd + d] : 0.f;
            acc[gi][e] = 0.f;
        }
    }
    for (int base = jlo + warp * U; base < jhi; base += NW * U) {
        float kk[U][EPL], vv[U][EPL];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = base + u;
            const bool ok = j < jhi;
            const float* kr = kb + (size_t)(ok ? j : jlo) * rs;
            const float* vr = vb + (size_t)(ok ? j : jlo) * rs;
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                int d = lane + 32 * e;
                bool in = ok && d < hd;
                if (LD == KV_NC) {
                    kk[u][e] = in ? __ldg(kr + d) : 0.f;
                    vv[u][e] = in ? __ldg(vr + d) : 0.f;
                } else if (LD == KV_CG) {
                    kk[u][e] = in ? __ldcg(kr + d) : 0.f;
                    vv[u][e] = in ? __ldcg(vr + d) : 0.f;
                } else {
                    kk[u][e] = in ? kr[d] : 0.f;
                    vv[u][e] = in ? vr[d] : 0.f;
                }
            }
        }
#pragma unroll
        for (int gi = 0; gi < GMAX; gi++) {
            if (gi < G) {
                float s[U];
                float mn = m[gi];
#pragma unroll
                for (int u = 0; u < U; u++) {
                    float p = 0.f;
#pragma unroll
                    for (int e = 0; e < EPL; e++) p = fmaf(qr[gi][e], kk[u][e], p);
                    s[u] = warp_sum(p) * scale;
                    if (softcap > 0.f) s[u] = softcap * tanhf(s[u] / softcap);
                    if (base + u < jhi) mn = fmaxf(mn, s[u]);
                }
                const float corr = expf(m[gi] - mn);
                float pe[U], psum = 0.f;
#pragma unroll
                for (int u = 0; u < U; u++) {
                    pe[u] = (base + u < jhi) ? expf(s[u] - mn) : 0.f;
                    psum += pe[u];
                }
                l[gi] = l[gi] * corr + psum;
#pragma unroll
                for (int e = 0; e < EPL; e++) {
                    float a = acc[gi][e] * corr;
#pragma unroll
                    for (int u = 0; u < U; u++) a = fmaf(vv[u][e], pe[u], a);
                    acc[gi][e] = a;
                }
                m[gi] = mn;
            }
        }
    }
#pragma unroll
    for (int gi = 0; gi < GMAX; gi++) {
        if (gi < G) {
            float* dst = sm + (size_t)(warp * G + gi) * W;
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                int d = lane + 32 * e;
                if (d < hd) dst[d] = acc[gi][e];
            }
            if (lane == 0) {
                dst[hd] = m[gi];
                dst[hd + 1] = l[gi];
            }
        }
    }
    attn_sync<NAMED, NW>();
    // merge the NW warp states (the merge rule of attention.wgsl:88-95): per
    // head, warp gi finds M = max_w m_w, the weights c_w = exp(m_w - M) and
    // L = sum_w l_w c_w (lane w holds warp w's state), so each output element
    // is a plain weighted sum of the NW accumulators
    float* cw = res + (size_t)G * W;  // [G][NW] merge weights
    for (int gi = warp; gi < G; gi += NW) {
        const float* st = sm + (size_t)gi * W;
        const float mw = lane < NW ? st[(size_t)lane * G * W + hd] : REF_NEG_INF;
        const float lw = lane < NW ? st[(size_t)lane * G * W + hd + 1] : 0.f;
        const float M = warp_max(mw);
        const float c = lane < NW ? expf(mw - M) : 0.f;
        const float L = warp_sum(lw * c);
        if (lane < NW) cw[gi * NW + lane] = c;
        if (lane == 0) {
            res[gi * W + hd] = M;
            res[gi * W + hd + 1] = L;
        }
    }
    attn_sync<NAMED, NW>();
    for (int i = threadIdx.x; i < G * hd; i += NW * 32) {
        int gi = i / hd, d = i - gi * hd;
        float A = 0.f;
#pragma unroll
        for (int w = 0; w < NW; w++) A = fmaf(sm[(size_t)(w * G + gi) * W + d], cw[gi * NW + w], A);
        res[gi * W + d] = A;
    }
    attn_sync<NAMED, NW>();
}

// After attn_core: with one active split, write the normalised output;
// otherwise publish this split's state to part[head][split][hd+2] and let the
// last CTA of the kv head merge the n_active splits (the counter resets itself
// to 0).  cwt is shared scratch of G*(n_active+1) floats for the merge weights.
static __device__ __noinline__ void attn_finish(const float* res, int G, int hd, int g, int split,
                                            int n_active, int n_splits_alloc,
                                            float* __restrict__ part,
                                            unsigned* __restrict__ counters,
                                            float* __restrict__ out, float* cwt,
                                            int nthreads = 0, bool named = false) {
    // nthreads: the threads that run it (0: the whole CTA, __syncthreads);
    // named: they synchronise with named barrier 1 (other warps do not)
    if (nthreads == 0) nthreads = blockDim.x;
    auto sync = [&]() {
        if (named)
            asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
        else
            __syncthreads();
    };
    const int W = hd + 2;
    if (n_active == 1) {
        for (int i = threadIdx.x; i < G * hd; i += nthreads) {
            int gi = i / hd, d = i - gi * hd;
            out[(size_t)(g * G + gi) * hd + d] = res[gi * W + d] * (1.0f / res[gi * W + hd + 1]);
        }
        return;
    }
    for (int i = threadIdx.x; i < G * W; i += nthreads) {
        int gi = i / W, d = i - gi * W;
        part[((size_t)(g * G + gi) * n_splits_alloc + split) * W + d] = res[i];
    }
    __threadfence();
    sync();
    __shared__ int s_last;
    if (threadIdx.x == 0) s_last = (atomicAdd(&counters[g], 1u) == (unsigned)n_active - 1);
    sync();
    if (!s_last) return;
    __threadfence();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // merge weights c_s = exp(M_s - M) and 1/L per head, one warp per head
    for (int gi = warp; gi < G; gi += (nthreads >> 5)) {
        const float* ph = part + (size_t)(g * G + gi) * n_splits_alloc * W;
        float M = REF_NEG_INF;
        for (int s = lane; s < n_active; s += 32) M = fmaxf(M, __ldcg(ph + (size_t)s * W + hd));
        M = warp_max(M);
        float L = 0.f;
        for (int s = lane; s < n_active; s += 32) {
            float c = expf(__ldcg(ph + (size_t)s * W + hd) - M);
            cwt[gi * (n_active + 1) + s] = c;
            L += __ldcg(ph + (size_t)s * W + hd + 1) * c;
        }
        L = warp_sum(L);
        if (lane == 0) cwt[gi * (n_active + 1) + n_active] = 1.0f / L;
    }
    sync();
    for (int i = threadIdx.x; i < G * hd; i += nthreads) {
        int gi = i / hd, d = i - gi * hd;
        const float* ph = part + (size_t)(g * G + gi) * n_splits_alloc * W + d;
        const float* c = cwt + gi * (n_active + 1);
        float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
        int s = 0;
        for (; s + 3 < n_active; s += 4) {
            a0 = fmaf(__ldcg(ph + (size_t)(s + 0) * W), c[s + 0], a0);
            a1 = fmaf(__ldcg(ph + (size_t)(s + 1) * W), c[s + 1], a1);
            a2 = fmaf(__ldcg(ph + (size_t)(s + 2) * W), c[s + 2], a2);
            a3 = fmaf(__ldcg(ph + (size_t)(s + 3) * W), c[s + 3], a3);
        }
        for (; s < n_active; s++) a0 = fmaf(__ldcg(ph + (size_t)s * W), c[s], a0);
        out[(size_t)(g * G + gi) * hd + d] = ((a0 + a1) + (a2 + a3)) * c[n_active];
    }
    sync();
    if (threadIdx.x == 0) counters[g] = 0;
}

}  // namespace cw
