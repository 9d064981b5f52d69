// cw_sample.cu -- the sampling kernels of the single-session step and the
// cw_sample op (rules and device code in cw_sample.cuh).
#include "cw_model.h"
#include "cw_sample.cuh"

namespace cw {

// After a decode step (whose finalize appended the argmax at toks[n-1] and
// made it the next input): replace it by the sampled token, and on an EOS
// token stop -- the token is not counted (wasm.rs:99-101), the session is
// marked stopped and later steps append nothing.
__global__ void __launch_bounds__(SMP_THREADS) k_sample_step(DevState* st,
                                                             const float* __restrict__ logits,
                                                             int n, const SampleParams* sp,
                                                             unsigned* __restrict__ toks) {
    __shared__ SmpShared S;
    const int np = st->n_produced;
    if (st->stopped) {  // stopped earlier: this step's token is dropped
        if (threadIdx.x == 0) st->n_produced = np - 1;
        return;
    }
    const SampleParams p = *sp;
    const unsigned amax = toks[np - 1];
    const unsigned t = sample_core(S, logits, n, p, (unsigned long long)(np - 1), amax);
    if (threadIdx.x == 0) {
        toks[np - 1] = t;
        st->token = t;
        bool eos = false;
        for (unsigned j = 0; j < p.n_eos; j++) eos |= p.eos[j] == t;
        if (eos) {
            st->stopped = 1;
            st->n_produced = np - 1;
        }
    }
}

// Standalone op: token for draw `draw` (argmax hint computed here).
__global__ void __launch_bounds__(SMP_THREADS) k_sample_op(const float* __restrict__ logits, int n,
                                                           SampleParams p,
                                                           unsigned long long draw,
                                                           unsigned* __restrict__ out) {
    __shared__ SmpShared S;
    __shared__ unsigned long long best[SMP_THREADS / 32];
    unsigned long long k = argmax_key_init();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const unsigned long long c = argmax_key(logits[i], (unsigned)i);
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
    __syncthreads();
    const unsigned t = sample_core(S, logits, n, p, draw, argmax_key_index(k));
    if (threadIdx.x == 0) *out = t;
}

// ---- host ----------------------------------------------------------------------
int sample_params_size() { return (int)sizeof(SampleParams); }

int sample_params_write(cw_session* s) {
    SampleParams p{};
    p.temperature = s->smp_temperature;
    p.top_k = s->smp_top_k;
    p.top_p = s->smp_top_p;
    p.seed = s->smp_seed;
    p.n_eos = (unsigned)s->eos.size();
    for (size_t i = 0; i < s->eos.size(); i++) p.eos[i] = s->eos[i];
    CW_CUDA(cudaMemcpyAsync(s->smp_dev, &p, sizeof p, cudaMemcpyHostToDevice, s->ctx->stream));
    CW_CUDA(cudaStreamSynchronize(s->ctx->stream));
    return CW_OK;
}

bool sample_active(const cw_session* s) { return s->smp_temperature > 0.f || !s->eos.empty(); }

int sample_enqueue(cw_session* s) {
    k_sample_step<<<1, SMP_THREADS, 0, s->ctx->stream>>>(s->st, s->logits, (int)s->m->info.vocab,
                                                         (const SampleParams*)s->smp_dev, s->toks);
    return check_launch("sample");
}

}  // namespace cw

using namespace cw;

extern "C" {

int cw_sample(cw_ctx* ctx, cw_buf logits, size_t n, float temperature, uint32_t top_k,
              float top_p, uint64_t seed, uint64_t draw, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out && n > 0 && n < (1ull << 31), CW_ERR_INVALID_ARG,
             "cw_sample: bad arguments");
    CW_CHECK(!(top_p < 0.f) && !(top_p > 1.f) && top_p == top_p, CW_ERR_INVALID_ARG,
             "cw_sample: top_p must lie in [0, 1]");
    BufEntry *el, *eo;
    CW_TRY(buf_get(ctx, logits, &el, n * 4, "cw_sample"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, 1, out, &eo));
    el = &ctx->bufs[logits];
    SampleParams p{};
    p.temperature = temperature;
    p.top_k = top_k;
    p.top_p = top_p;
    p.seed = seed;
    OpScope scope(ctx, "sample");
    k_sample_op<<<1, SMP_THREADS, 0, ctx->stream>>>((const float*)el->ptr, (int)n, p, draw,
                                                    (unsigned*)eo->ptr);
    return check_launch("sample");
}

}  // extern "C"
