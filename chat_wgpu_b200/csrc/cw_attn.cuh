// cw_attn.cuh -- split-KV single-query attention core shared by the
// stand-alone op (cw_attention) and the fused decode kernel.
//
// Semantics follow chat-wgpu src/kernels/attention.wgsl:23-96: scores
// s = scale * (q . k_j), an online softmax (running max m, denominator l,
// rescaled accumulator), GQA head h -> kv head h / (n_heads / n_kv).
// Work split: one CTA per (key range, kv head); the CTA's 4 warps take keys
// j = lo + w, lo + w + 4, ... and each warp keeps an online-softmax state for
// every query head of the group (GQA: K/V rows are read once per group).
// Lane l holds head dims l, l+32, ... so each key row is one coalesced
// 128-byte read per 32 dims.
#pragma once

#include "cw_device.cuh"

namespace cw {

constexpr float REF_NEG_INF = -3.402823e38f;  // attention.wgsl:27

// Shared memory floats needed by attn_core for G heads of dim hd.
__host__ __device__ constexpr size_t attn_smem_floats(int G, int hd) {
    return (size_t)5 * G * (hd + 2);
}

// Computes, for the G query heads in qg[G][hd] (global or shared memory),
// the un-normalised attention state over keys [jlo, jhi) of one kv head
// (rows kb + j*rs, vb + j*rs).  On return res[gi*(hd+2) + d] holds the
// accumulator A, res[.. + hd] the max M, res[.. + hd + 1] the denominator L
// (all threads of the 128-thread CTA call it; it ends with __syncthreads()).
// NC selects the read-only (non-coherent) load path; it must be false when
// the calling kernel itself wrote K/V rows it then reads.
template <int EPL, int GMAX, bool NC = true>
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
    for (int j = jlo + warp; j < jhi; j += 4) {
        const float* kr = kb + (size_t)j * rs;
        const float* vr = vb + (size_t)j * rs;
        float kk[EPL], vv[EPL];
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            int d = lane + 32 * e;
            if (NC) {
                kk[e] = d < hd ? __ldg(kr + d) : 0.f;
                vv[e] = d < hd ? __ldg(vr + d) : 0.f;
            } else {
                kk[e] = d < hd ? kr[d] : 0.f;
                vv[e] = d < hd ? vr[d] : 0.f;
            }
        }
#pragma unroll
        for (int gi = 0; gi < GMAX; gi++) {
            if (gi < G) {
                float p = 0.f;
#pragma unroll
                for (int e = 0; e < EPL; e++) p = fmaf(qr[gi][e], kk[e], p);
                float s = warp_sum(p) * scale;
                if (softcap > 0.f) s = softcap * tanhf(s / softcap);
                float mn = fmaxf(m[gi], s);
                float corr = expf(m[gi] - mn);
                float pe = expf(s - mn);
                l[gi] = l[gi] * corr + pe;
#pragma unroll
                for (int e = 0; e < EPL; e++) acc[gi][e] = acc[gi][e] * corr + vv[e] * pe;
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
    __syncthreads();
    // merge the 4 warp states (attention.wgsl:88-95 merge rule)
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        int gi = i / hd, d = i - gi * hd;
        float M = REF_NEG_INF;
#pragma unroll
        for (int w = 0; w < 4; w++) M = fmaxf(M, sm[(size_t)(w * G + gi) * W + hd]);
        float L = 0.f, A = 0.f;
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const float* src = sm + (size_t)(w * G + gi) * W;
            float c = expf(src[hd] - M);
            L += src[hd + 1] * c;
            A += src[d] * c;
        }
        res[gi * W + d] = A;
        if (d == 0) {
            res[gi * W + hd] = M;
            res[gi * W + hd + 1] = L;
        }
    }
    __syncthreads();
}

// After attn_core: either write the normalised output (one split), or
// publish this split's state to part[head][split][hd+2] and let the last CTA
// of the kv head merge all splits (counter self-resets to 0).
__device__ __forceinline__ void attn_finish(const float* res, int G, int hd, int g, int split,
                                            int n_splits, float* __restrict__ part,
                                            unsigned* __restrict__ counters,
                                            float* __restrict__ out) {
    const int W = hd + 2;
    if (n_splits == 1) {
        for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
            int gi = i / hd, d = i - gi * hd;
            out[(size_t)(g * G + gi) * hd + d] = res[gi * W + d] * (1.0f / res[gi * W + hd + 1]);
        }
        return;
    }
    for (int i = threadIdx.x; i < G * W; i += blockDim.x) {
        int gi = i / W, d = i - gi * W;
        part[((size_t)(g * G + gi) * n_splits + split) * W + d] = res[i];
    }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (threadIdx.x == 0) s_last = (atomicAdd(&counters[g], 1u) == (unsigned)n_splits - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
        int gi = i / hd, d = i - gi * hd;
        const float* ph = part + (size_t)(g * G + gi) * n_splits * W;
        float M = REF_NEG_INF;
        for (int s = 0; s < n_splits; s++) M = fmaxf(M, __ldcg(ph + (size_t)s * W + hd));
        float L = 0.f, A = 0.f;
        for (int s = 0; s < n_splits; s++) {
            float c = expf(__ldcg(ph + (size_t)s * W + hd) - M);
            L += __ldcg(ph + (size_t)s * W + hd + 1) * c;
            A += __ldcg(ph + (size_t)s * W + d) * c;
        }
        out[(size_t)(g * G + gi) * hd + d] = A * (1.0f / L);
    }
    __syncthreads();
    if (threadIdx.x == 0) counters[g] = 0;
}

// Key range of split `split` out of n_splits over the (windowed) prefix
// [j0, seq): j0 = seq - window for a sliding-window layer.
__device__ __forceinline__ void attn_range(int seq, int window, int split, int n_splits, int* jlo,
                                           int* jhi) {
    int j0 = (window > 0 && seq > window) ? seq - window : 0;
    int span = seq - j0;
    int per = (span + n_splits - 1) / n_splits;
    *jlo = min(seq, j0 + split * per);
    *jhi = min(seq, *jlo + per);
}

}  // namespace cw
