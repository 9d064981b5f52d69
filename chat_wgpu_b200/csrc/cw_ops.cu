// cw_ops.cu -- the per-op wrappers of chat-wgpu src/kernels/*.rs: rmsnorm,
// rope, attention, add, swiglu/geglu, argmax.  Each entry point takes and
// returns buffer handles like the Rust wrapper it replaces and enqueues on
// the context stream.
#include <algorithm>

#include "cw_attn.cuh"
#include "cw_common.h"
#include "cw_device.cuh"
#include "cw_ops.h"

namespace cw {

// ---- rmsnorm: norm.wgsl:20-56 -------------------------------------------
__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; i++) t += red[i];
    return t;
}

__global__ void __launch_bounds__(256) k_rmsnorm(const float* __restrict__ x,
                                                 const float* __restrict__ w,
                                                 float* __restrict__ y, int dim, float eps,
                                                 int unit) {
    __shared__ float red[32];
    const float* xr = x + (size_t)blockIdx.x * dim;
    float* yr = y + (size_t)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum(ss, red);
    float inv = 1.0f / sqrtf(ss / (float)dim + eps);
    for (int i = threadIdx.x; i < dim; i += blockDim.x) {
        float g = unit ? 1.0f + w[i] : w[i];
        yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), g);
    }
}

int launch_rmsnorm(cw_ctx* ctx, const float* x, const float* w, float* y, int rows, int dim,
                   float eps, int unit) {
    int threads = std::min(256, std::max(32, ((dim + 3) / 4 + 31) / 32 * 32));
    k_rmsnorm<<<rows, threads, 0, ctx->stream>>>(x, w, y, dim, eps, unit);
    return check_launch("rmsnorm");
}

// ---- rope: rope.wgsl:25-34 -------------------------------------------------
// freq = f32(pos) * inv_freq[i] with inv_freq from the host table (the same
// f32 pow the shader evaluates); accurate sincosf; two roundings per term.
__global__ void k_rope(const float* __restrict__ x, float* __restrict__ y, int rows, int hd,
                       const float* __restrict__ inv_freq, int pos) {
    int half = hd / 2;
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= rows * half) {
        // odd head_dim: the unrotated last element is carried through
        if ((hd & 1) && idx < rows * half + rows) {
            int r = idx - rows * half;
            y[(size_t)r * hd + hd - 1] = x[(size_t)r * hd + hd - 1];
        }
        return;
    }
    int r = idx / half, i = idx - r * half;
    float freq = __fmul_rn((float)pos, inv_freq[i]);
    float s, c;
    sincosf(freq, &s, &c);
    size_t base = (size_t)r * hd;
    float lo = x[base + i], hi = x[base + i + half];
    y[base + i] = __fsub_rn(__fmul_rn(lo, c), __fmul_rn(hi, s));
    y[base + i + half] = __fadd_rn(__fmul_rn(hi, c), __fmul_rn(lo, s));
}

int launch_rope(cw_ctx* ctx, const float* x, float* y, int rows, int hd, int pos, float theta) {
    const float* tbl;
    CW_TRY(rope_table(ctx, (uint32_t)hd, theta, &tbl));
    int n = rows * (hd / 2) + rows;
    k_rope<<<(n + 127) / 128, 128, 0, ctx->stream>>>(x, y, rows, hd, tbl, pos);
    return check_launch("rope");
}

// ---- attention: attention.wgsl:23-96 ----------------------------------------
template <int EPL, int GMAX>
__global__ void __launch_bounds__(128) k_attention(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    float* __restrict__ out, int n_heads, int n_kv, int seq, int hd, float scale, float softcap,
    int window, long head_stride, long row_stride, int n_splits, float* __restrict__ part,
    unsigned* __restrict__ counters) {
    extern __shared__ float sm[];
    const int G = n_heads / n_kv;
    const int g = blockIdx.y, split = blockIdx.x;
    const int n_active = attn_active_splits(attn_span(seq, window), n_splits);
    if (split >= n_active) return;
    int jlo, jhi;
    attn_range(seq, window, split, n_active, &jlo, &jhi);
    float* res = sm + 4 * G * (hd + 2);
    float* cwt = sm + 5 * G * (hd + 2);
    attn_core<EPL, GMAX>(q + (size_t)g * G * hd, G, hd, k + g * head_stride, v + g * head_stride,
                         row_stride, jlo, jhi, scale, softcap, sm, res);
    attn_finish(res, G, hd, g, split, n_active, n_splits, part, counters, out, cwt);
}

template <int EPL>
static int attn_dispatch_g(int G, dim3 grid, size_t smem, cudaStream_t st, const float* q,
                           const float* k, const float* v, float* out, int n_heads, int n_kv,
                           int seq, int hd, float scale, float softcap, int window, long hs, long rs,
                           int n_splits, float* part, unsigned* counters) {
#define CW_ATTN_LAUNCH(GM)                                                                     \
    do {                                                                                       \
        if (smem > 48 * 1024)                                                                  \
            CW_CUDA(cudaFuncSetAttribute(k_attention<EPL, GM>,                                 \
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,          \
                                         (int)smem));                                          \
        k_attention<EPL, GM><<<grid, 128, smem, st>>>(q, k, v, out, n_heads, n_kv, seq, hd,    \
                                                      scale, softcap, window, hs, rs,          \
                                                      n_splits, part, counters);               \
    } while (0)
    if (G <= 1) CW_ATTN_LAUNCH(1);
    else if (G <= 2) CW_ATTN_LAUNCH(2);
    else if (G <= 4) CW_ATTN_LAUNCH(4);
    else CW_ATTN_LAUNCH(8);
#undef CW_ATTN_LAUNCH
    return check_launch("attention");
}

int attention_splits_for(int sm_count, int span, int n_kv);

int attention_splits(cw_ctx* ctx, int span, int n_kv) {
    return attention_splits_for(ctx->sm_count, span, n_kv);
}

int attention_splits_for(int sm_count, int span, int n_kv) {
    int by_sm = std::max(1, 2 * sm_count / std::max(1, n_kv));
    return attn_active_splits(span, by_sm);
}

int launch_attention_raw(cudaStream_t st, const float* q, const float* k, const float* v,
                         float* out, int n_heads, int n_kv, int seq, int hd, float softcap,
                         int window, long head_stride, long row_stride, int n_splits, float* part,
                         unsigned* counters) {
    const int G = n_heads / n_kv;
    const float scale = powf((float)hd, -0.5f);  // attention.rs:18
    size_t smem = attn_smem_floats(G, hd, n_splits) * sizeof(float);
    dim3 grid(n_splits, n_kv);
    int epl = (hd + 31) / 32;
    auto go = [&](auto tag) -> int {
        constexpr int E = decltype(tag)::value;
        return attn_dispatch_g<E>(G, grid, smem, st, q, k, v, out, n_heads, n_kv, seq, hd, scale,
                                  softcap, window, head_stride, row_stride, n_splits, part,
                                  counters);
    };
    if (epl <= 1) return go(std::integral_constant<int, 1>());
    if (epl <= 2) return go(std::integral_constant<int, 2>());
    if (epl <= 4) return go(std::integral_constant<int, 4>());
    return go(std::integral_constant<int, 8>());
}

int launch_attention(cw_ctx* ctx, const float* q, const float* k, const float* v, float* out,
                     int n_heads, int n_kv, int seq, int hd, float softcap, int window,
                     long head_stride, long row_stride, int n_splits, float* part) {
    CW_TRY(ensure_counters(ctx, (size_t)n_kv));
    return launch_attention_raw(ctx->stream, q, k, v, out, n_heads, n_kv, seq, hd, softcap, window,
                                head_stride, row_stride, n_splits, part, ctx->d_counters);
}

// ---- elementwise: ewise.wgsl:9-13, glu.wgsl:22-32 ----------------------------
__global__ void k_add(const float* __restrict__ a, const float* __restrict__ b,
                      float* __restrict__ c, size_t n) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) c[i] = a[i] + b[i];
}

__device__ __forceinline__ float silu_ref(float x) { return x / (1.0f + expf(-x)); }
__device__ __forceinline__ float gelu_ref(float x) {
    const float c = 0.7978845608028654f;
    return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
}

__global__ void k_glu(const float* __restrict__ g, const float* __restrict__ u,
                      float* __restrict__ o, size_t n, int geglu) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float a = geglu ? gelu_ref(g[i]) : silu_ref(g[i]);
    o[i] = a * u[i];
}

// ---- argmax: argmax.wgsl:18-55 -----------------------------------------------
__device__ __forceinline__ unsigned long long u64max(unsigned long long a, unsigned long long b) {
    return a > b ? a : b;
}

__global__ void __launch_bounds__(256) k_argmax_partial(const float* __restrict__ x, size_t n,
                                                        unsigned long long* __restrict__ part) {
    __shared__ unsigned long long red[8];
    unsigned long long best = argmax_key_init();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        best = u64max(best, argmax_key(x[i], (unsigned)i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = u64max(best, __shfl_xor_sync(FULL, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < (int)(blockDim.x >> 5); i++) best = u64max(best, red[i]);
        part[blockIdx.x] = best;
    }
}

__global__ void k_argmax_final(const unsigned long long* __restrict__ part, int nparts,
                               unsigned* __restrict__ out) {
    unsigned long long best = argmax_key_init();
    for (int i = threadIdx.x; i < nparts; i += 32) best = u64max(best, part[i]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = u64max(best, __shfl_xor_sync(FULL, best, o));
    if (threadIdx.x == 0) out[0] = argmax_key_index(best);
}

}  // namespace cw

using namespace cw;

extern "C" {

static int norm_op(cw_ctx* ctx, cw_buf x, cw_buf w, size_t rows, size_t dim, float eps, int unit,
                   cw_buf* out, const char* name) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "%s: bad arguments", name);
    CW_CHECK(rows > 0 && dim > 0 && rows < (1u << 31), CW_ERR_INVALID_ARG, "%s: bad shape", name);
    BufEntry *ex, *ew, *ey;
    CW_TRY(buf_get(ctx, x, &ex, rows * dim * 4, name));
    CW_TRY(buf_get(ctx, w, &ew, dim * 4, name));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, rows * dim, out, &ey));
    OpScope scope(ctx, name);
    return launch_rmsnorm(ctx, (const float*)ex->ptr, (const float*)ew->ptr, (float*)ey->ptr,
                          (int)rows, (int)dim, eps, unit);
}

int cw_rmsnorm(cw_ctx* ctx, cw_buf x, cw_buf w, size_t rows, size_t dim, float eps, cw_buf* out) {
    return norm_op(ctx, x, w, rows, dim, eps, 0, out, "rmsnorm");
}

int cw_rmsnorm_unit(cw_ctx* ctx, cw_buf x, cw_buf w, size_t rows, size_t dim, float eps,
                    cw_buf* out) {
    return norm_op(ctx, x, w, rows, dim, eps, 1, out, "rmsnorm_unit");
}

int cw_rope(cw_ctx* ctx, cw_buf x, size_t rows, size_t head_dim, size_t pos, float theta,
            cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_rope: bad arguments");
    CW_CHECK(rows > 0 && head_dim > 0 && rows * head_dim < (1u << 31) && pos < (1u << 31),
             CW_ERR_INVALID_ARG, "cw_rope: bad shape");
    BufEntry *ex, *ey;
    CW_TRY(buf_get(ctx, x, &ex, rows * head_dim * 4, "cw_rope"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, rows * head_dim, out, &ey));
    OpScope scope(ctx, "rope");
    return launch_rope(ctx, (const float*)ex->ptr, (float*)ey->ptr, (int)rows, (int)head_dim,
                       (int)pos, theta);
}

int cw_attention_ext(cw_ctx* ctx, cw_buf q, cw_buf k, cw_buf v, size_t n_heads, size_t n_kv,
                     size_t seq, size_t head_dim, float softcap, uint32_t window, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_attention: bad arguments");
    CW_CHECK(n_heads > 0 && n_kv > 0 && n_heads % n_kv == 0 && n_heads / n_kv <= 8,
             CW_ERR_INVALID_ARG, "cw_attention: n_heads=%zu n_kv=%zu (need n_kv | n_heads, group <= 8)",
             n_heads, n_kv);
    CW_CHECK(head_dim > 0 && head_dim <= 256, CW_ERR_INVALID_ARG,
             "cw_attention: head_dim %zu (1..256, as the reference's q_sh[256])", head_dim);
    CW_CHECK(seq > 0 && seq < (1u << 30), CW_ERR_INVALID_ARG, "cw_attention: seq must be >= 1");
    BufEntry *eq, *ek, *ev, *eo;
    CW_TRY(buf_get(ctx, q, &eq, n_heads * head_dim * 4, "cw_attention(q)"));
    CW_TRY(buf_get(ctx, k, &ek, seq * n_kv * head_dim * 4, "cw_attention(k)"));
    CW_TRY(buf_get(ctx, v, &ev, seq * n_kv * head_dim * 4, "cw_attention(v)"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, n_heads * head_dim, out, &eo));
    int j0 = (window > 0 && seq > window) ? (int)(seq - window) : 0;
    int n_splits = attention_splits(ctx, (int)seq - j0, (int)n_kv);
    float* part = nullptr;
    if (n_splits > 1) {
        cw_buf pb;
        BufEntry* ep;
        CW_TRY(arena_get(ctx, n_heads * n_splits * (head_dim + 2), &pb, &ep));
        part = (float*)ep->ptr;
    }
    OpScope scope(ctx, "attention");
    return launch_attention(ctx, (const float*)eq->ptr, (const float*)ek->ptr,
                            (const float*)ev->ptr, (float*)eo->ptr, (int)n_heads, (int)n_kv,
                            (int)seq, (int)head_dim, softcap, (int)window, (long)head_dim,
                            (long)(n_kv * head_dim), n_splits, part);
}

int cw_attention(cw_ctx* ctx, cw_buf q, cw_buf k, cw_buf v, size_t n_heads, size_t n_kv,
                 size_t seq, size_t head_dim, cw_buf* out) {
    return cw_attention_ext(ctx, q, k, v, n_heads, n_kv, seq, head_dim, 0.0f, 0, out);
}

int cw_add(cw_ctx* ctx, cw_buf a, cw_buf b, size_t n, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out && n > 0, CW_ERR_INVALID_ARG, "cw_add: bad arguments");
    BufEntry *ea, *eb, *ec;
    CW_TRY(buf_get(ctx, a, &ea, n * 4, "cw_add(a)"));
    CW_TRY(buf_get(ctx, b, &eb, n * 4, "cw_add(b)"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, n, out, &ec));
    OpScope scope(ctx, "ewise_add");
    k_add<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
        (const float*)ea->ptr, (const float*)eb->ptr, (float*)ec->ptr, n);
    return check_launch("add");
}

static int glu_op(cw_ctx* ctx, cw_buf gate, cw_buf up, size_t n, cw_buf* out, int geglu,
                  const char* name) {
    clear_error();
    CW_CHECK(ctx && out && n > 0, CW_ERR_INVALID_ARG, "%s: bad arguments", name);
    BufEntry *eg, *eu, *eo;
    CW_TRY(buf_get(ctx, gate, &eg, n * 4, name));
    CW_TRY(buf_get(ctx, up, &eu, n * 4, name));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, n, out, &eo));
    OpScope scope(ctx, name);
    k_glu<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
        (const float*)eg->ptr, (const float*)eu->ptr, (float*)eo->ptr, n, geglu);
    return check_launch(name);
}

int cw_swiglu(cw_ctx* ctx, cw_buf gate, cw_buf up, size_t n, cw_buf* out) {
    return glu_op(ctx, gate, up, n, out, 0, "swiglu");
}

int cw_geglu(cw_ctx* ctx, cw_buf gate, cw_buf up, size_t n, cw_buf* out) {
    return glu_op(ctx, gate, up, n, out, 1, "geglu");
}

int cw_argmax(cw_ctx* ctx, cw_buf logits, size_t n, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out && n > 0 && n < (1ull << 32), CW_ERR_INVALID_ARG, "cw_argmax: bad arguments");
    BufEntry *el, *eo, *ep;
    CW_TRY(buf_get(ctx, logits, &el, n * 4, "cw_argmax"));
    cudaSetDevice(ctx->device);
    CW_TRY(arena_get(ctx, 1, out, &eo));
    int nparts = (int)std::min<size_t>((n + 2047) / 2048, (size_t)ctx->sm_count * 2);
    nparts = std::max(nparts, 1);
    cw_buf pb;
    CW_TRY(arena_get(ctx, (size_t)nparts * 2, &pb, &ep));
    el = &ctx->bufs[logits];
    eo = &ctx->bufs[*out];
    OpScope scope(ctx, "argmax");
    k_argmax_partial<<<nparts, 256, 0, ctx->stream>>>((const float*)el->ptr, n,
                                                      (unsigned long long*)ep->ptr);
    k_argmax_final<<<1, 32, 0, ctx->stream>>>((const unsigned long long*)ep->ptr, nparts,
                                              (unsigned*)eo->ptr);
    return check_launch("argmax");
}

}  // extern "C"
