// cw_sample.cuh -- sampling and stop conditions after the LM head (device code
// shared by the single-session step, cw_sample.cu, and the co-batched step).
//
// The reference decodes greedily (argmax, src/kernels/argmax.wgsl) and stops
// its browser chat loop when the argmax is an EOS id, before emitting it
// (src/wasm.rs:48-51,99-101); temperature is accepted but unused there
// (wasm.rs:57,63) and temperature / top-k / top-p are on its roadmap
// (ROADMAP.md:56-57).  This file adds them on the device, so a decode step
// still needs no logits readback:
//
//   temperature T <= 0        greedy: the step's argmax (lowest index on ties)
//   T > 0                     w_i = exp((l_i - max) / T), NaN logits excluded
//   top_k > 0                 keep logits >= the k-th largest logit (ties kept)
//   top_p < 1                 of those, keep w_i >= tau, tau the largest value
//                             whose kept mass sum_{w >= tau} w reaches top_p of
//                             the total (the nucleus; ties kept)
//   draw                      u = splitmix64(seed ^ (draw + 1) * 0x9E3779B97F4A7C15)
//                             >> 11 (53 bits); target = floor(u * Z / 2^53) with
//                             Z = sum of the kept masses; the token is the first
//                             index i whose inclusive prefix sum exceeds target
//
// Masses are fixed point (w * 2^40 truncated to u64), so every sum, the
// nucleus threshold and the draw are exact and order-independent; thresholds
// are found by 4-pass radix selection over the order-preserving 32-bit keys.
// One CTA of 1024 threads.
#pragma once

#include <stdint.h>

#include "cw_common.h"
#include "cw_device.cuh"

namespace cw {

constexpr int SMP_THREADS = 1024;
constexpr double SMP_FIX = 1099511627776.0;  // 2^40

struct SampleParams {
    float temperature;
    unsigned top_k;
    float top_p;
    unsigned n_eos;
    unsigned long long seed;
    unsigned eos[CW_MAX_EOS];
};

__device__ __forceinline__ unsigned long long smp_mix(unsigned long long x) {  // splitmix64
    x += 0x9E3779B97F4A7C15ull;
    x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
    x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
    return x ^ (x >> 31);
}

__device__ __forceinline__ unsigned smp_key(float v) {  // NaN sorts below everything
    return v != v ? 0u : f32_order_key(v);
}

struct SmpShared {
    unsigned long long hist[256];
    unsigned long long part[SMP_THREADS / 32];
    unsigned prefix;
    unsigned long long remain;
    unsigned token;
};

// Largest key tau with sum over {i: key_i >= tau} of weight_i >= need, where
// weight_i = 1 (count) or the fixed-point mass; keys are given by `keyf(i)`
// (0 = excluded).
template <class KeyF, class WF>
__device__ inline unsigned smp_select(SmpShared& S, int n, unsigned long long need, KeyF keyf, WF wf) {
    const int tid = threadIdx.x;
    unsigned prefix = 0, mask = 0;
    unsigned long long remain = need;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int b = tid; b < 256; b += blockDim.x) S.hist[b] = 0ull;
        __syncthreads();
        for (int i = tid; i < n; i += blockDim.x) {
            const unsigned k = keyf(i);
            if (k != 0u && (k & mask) == prefix) {
                const unsigned long long w = wf(i);
                if (w) atomicAdd(&S.hist[(k >> shift) & 255u], w);
            }
        }
        __syncthreads();
        if (tid == 0) {
            unsigned long long cum = 0ull;
            int b = 255;
            for (; b > 0; b--) {
                if (cum + S.hist[b] >= remain) break;
                cum += S.hist[b];
            }
            S.prefix = prefix | ((unsigned)b << shift);
            S.remain = remain - cum;
        }
        __syncthreads();
        prefix = S.prefix;
        remain = S.remain;
        mask |= 255u << shift;
        __syncthreads();
    }
    return prefix;
}

// Exclusive prefix sum over the CTA's threads (thread order) and the total.
__device__ __forceinline__ unsigned long long smp_scan(SmpShared& S, unsigned long long v,
                                                       unsigned long long* total) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
    unsigned long long x = v;
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) S.part[warp] = x;
    __syncthreads();
    if (warp == 0) {
        unsigned long long w = lane < nw ? S.part[lane] : 0ull;
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned long long y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        if (lane < nw) S.part[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    const unsigned long long before = (warp ? S.part[warp - 1] : 0ull) + x - v;
    *total = S.part[nw - 1];
    __syncthreads();
    return before;
}

// Token for one draw from logits[0, n) under `sp`; `amax` = index of the max
// logit (the greedy answer).  All threads of the CTA call it.
__device__ inline unsigned sample_core(SmpShared& S, const float* __restrict__ logits, int n,
                                const SampleParams& sp, unsigned long long draw, unsigned amax) {
    const int tid = threadIdx.x;
    if (!(sp.temperature > 0.f)) return amax;  // greedy (logits may be a vocabulary shard)
    const float M = logits[amax];
    if (M != M) return amax;
    const float invT = 1.0f / sp.temperature;
    // top-k threshold over the logits
    unsigned tk = 0u;
    if (sp.top_k > 0 && sp.top_k < (unsigned)n)
        tk = smp_select(
            S, n, sp.top_k, [&](int i) { return smp_key(logits[i]); },
            [&](int) { return 1ull; });
    // relative probability w_i (0 = excluded) and its fixed-point mass
    auto wf = [&](int i) -> float {
        const float l = logits[i];
        const unsigned k = smp_key(l);
        if (k == 0u || k < tk) return 0.f;
        return expf((l - M) * invT);
    };
    auto mass = [](float w) { return (unsigned long long)((double)w * SMP_FIX); };
    // nucleus threshold over the w (keys of positive floats order like the floats)
    unsigned tp = 0u;
    if (sp.top_p < 1.0f) {
        unsigned long long own = 0ull, total = 0ull;
        for (int i = tid; i < n; i += blockDim.x) own += mass(wf(i));
        smp_scan(S, own, &total);
        unsigned long long need = (unsigned long long)((double)sp.top_p * (double)total);
        if (need == 0ull) need = 1ull;
        tp = smp_select(
            S, n, need,
            [&](int i) {
                const float w = wf(i);
                return mass(w) ? f32_order_key(w) : 0u;
            },
            [&](int i) { return mass(wf(i)); });
    }
    auto kept = [&](int i) -> unsigned long long {
        const float w = wf(i);
        const unsigned long long m = mass(w);
        if (!m || (tp && f32_order_key(w) < tp)) return 0ull;
        return m;
    };
    // per-thread contiguous chunks, exclusive scan of the chunk sums, then the
    // chunk holding the target scans its elements in index order
    const int chunk = (n + blockDim.x - 1) / blockDim.x;
    const int i0 = min(n, tid * chunk), i1 = min(n, i0 + chunk);
    unsigned long long own = 0ull;
    for (int i = i0; i < i1; i++) own += kept(i);
    unsigned long long Z = 0ull;
    unsigned long long acc = smp_scan(S, own, &Z);
    if (tid == 0) S.token = amax;
    __syncthreads();
    const unsigned long long u = smp_mix(sp.seed ^ ((draw + 1ull) * 0x9E3779B97F4A7C15ull)) >> 11;
    const unsigned long long target = __umul64hi(u << 11, Z);  // floor(u * Z / 2^53)
    if (Z > 0ull && own > 0ull && acc <= target && target < acc + own) {
        for (int i = i0; i < i1; i++) {
            acc += kept(i);
            if (acc > target) {
                S.token = (unsigned)i;
                break;
            }
        }
    }
    __syncthreads();
    return S.token;
}

}  // namespace cw
