// cw_common.h -- internal declarations shared by the libchatcuda.so sources.
//
// The context mirrors chat-wgpu's GpuContext (src/context.rs): a device and a
// stream, a buffer table, the per-frame arena (empty()/reset_frame()), and a
// per-op timing profiler (src/profile.rs) built on CUDA events.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include <map>
#include <string>
#include <unordered_map>
#include <utility>
#include <vector>

#include "../../include/chatcuda.h"

namespace cw {

// ---- errors ---------------------------------------------------------------
// Thread-local message for cw_last_error(); set_error returns the status so
// call sites can `return set_error(...)`.
int set_error(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
void clear_error();

#define CW_CUDA(call)                                                              \
    do {                                                                           \
        cudaError_t e_ = (call);                                                   \
        if (e_ != cudaSuccess)                                                     \
            return ::cw::set_error(e_ == cudaErrorMemoryAllocation ? CW_ERR_OOM    \
                                                                   : CW_ERR_CUDA,  \
                                   "%s: %s (%s:%d)", #call, cudaGetErrorString(e_),\
                                   __FILE__, __LINE__);                            \
    } while (0)

#define CW_CHECK(cond, status, ...)                                                \
    do {                                                                           \
        if (!(cond)) return ::cw::set_error((status), __VA_ARGS__);                \
    } while (0)

#define CW_TRY(expr)                                                               \
    do {                                                                           \
        int s_ = (expr);                                                           \
        if (s_ != CW_OK) return s_;                                                \
    } while (0)

// Device-side status word written by bounded waits (never a trap).
enum DeviceStatus : int { DEV_OK = 0, DEV_TIMEOUT = 1, DEV_BAD_INPUT = 2 };

enum BufKind : int { BUF_STORAGE = 0, BUF_PERSISTENT = 1, BUF_ARENA = 2 };

struct BufEntry {
    void* ptr = nullptr;
    size_t nbytes = 0;
    int kind = BUF_STORAGE;
    // Set for packed Q4_0 weights: rows x in_f and the byte offset of the f16
    // scale plane (the nibble plane starts at 0).
    size_t rows = 0, in_f = 0, scale_off = 0;
    bool q4_0 = false;
    // Set for a Q6_K weight split for the streaming GEMV (cw_q6_k_split):
    // [rows][in_f/256][208] payload, f16 d plane at scale_off.
    bool q6k_split = false;
    // Set for a Q8_0 weight split for the streaming GEMV (cw_q8_0_split):
    // [rows][in_f/32][32] codes, f16 scale plane at scale_off.
    bool q8_split = false;
};

struct ProfRec {
    const char* name;
    cudaEvent_t start, stop;
};

}  // namespace cw

struct cw_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    int sm_count = 0;
    int clock_khz = 1;  // max SM clock (profile cycle conversion)
    int max_smem_optin = 0;
    int smem_per_sm = 0;
    size_t l2_bytes = 0;
    std::string backend;

    std::unordered_map<uint64_t, cw::BufEntry> bufs;
    uint64_t next_id = 1;
    // arena[slot] = (len in f32 elements, buffer id) -- context.rs:42-47
    std::vector<std::pair<size_t, uint64_t>> arena;
    size_t cursor = 0;

    // launch model kernels with programmatic dependent launch (PDL)
    bool pdl = true;

    // profiler (context.rs:53-56, profile.rs)
    bool profiling = false;
    std::vector<cw::ProfRec> prof;
    std::vector<cudaEvent_t> event_pool;

    // device status word (DeviceStatus) and zero-initialised per-head
    // completion counters used by the split-KV attention combine.
    int* d_status = nullptr;
    unsigned* d_counters = nullptr;
    size_t n_counters = 0;

    // RoPE inverse-frequency tables keyed by (head_dim, theta bits).
    std::map<std::pair<uint32_t, uint32_t>, float*> rope_tables;

    // grow-only scratch of the prefill GEMM op (split f16 operands)
    void* gemm_scratch = nullptr;
    size_t gemm_scratch_bytes = 0;
};

namespace cw {

// buffer helpers (cw_context.cu)
int buf_get(cw_ctx* ctx, cw_buf b, BufEntry** out, size_t min_bytes, const char* what);
int buf_new(cw_ctx* ctx, size_t nbytes, int kind, cw_buf* out, BufEntry** entry = nullptr);
int arena_get(cw_ctx* ctx, size_t len_f32, cw_buf* out, BufEntry** entry = nullptr);
int check_launch(const char* what);
int check_device_status(cw_ctx* ctx);

// A profiler scope: records a start/stop event pair around the launches made
// while it is alive, labelled with the op name (context.rs:302-328).
struct OpScope {
    cw_ctx* ctx;
    const char* name;
    cudaEvent_t start = nullptr, stop = nullptr;
    unsigned flags = 0;
    OpScope(cw_ctx* c, const char* n);
    ~OpScope();
};

// RoPE table for (head_dim, theta): inv_freq[i] = theta^(-2i/head_dim)
// computed on the host in f32 exactly as rope.wgsl:26-27 writes it.
int rope_table(cw_ctx* ctx, uint32_t head_dim, float theta, const float** out);

// zeroed counters for the attention combine; grows on demand (syncs).
int ensure_counters(cw_ctx* ctx, size_t n);

// Kernel launch on the context stream, with programmatic stream serialisation
// when `pdl` (the kernel may start before its predecessor finishes, up to its
// griddepcontrol.wait).
template <typename... KArgs, typename... Args>
inline int launch_pdl(cw_ctx* ctx, bool pdl, void (*kern)(KArgs...), dim3 grid, dim3 block,
                      size_t smem, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    CW_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
    return CW_OK;
}

// cw_gemm.cu: the tcgen05 prefill GEMM, Y[M,N] (=|+=) X[M,K] W[N,K]^T (+bias)
// over split f16 operands (xh/xl [M,K], wh/wl [N,K]; see cw_gemm.cuh).
// ws (may be null): workspace for split-K partial tiles when M is small and N
// has few tiles; the split is chosen to fit ws_bytes.
int gemm_x3(cw_ctx* ctx, const void* xh, const void* xl, const void* wh, const void* wl, int M,
            int N, int K, float* y, int ldy, const float* bias, int epi, float* ws = nullptr,
            size_t ws_bytes = 0, bool pdl = false);
// The same product with W as packed Q4_0 tile records (q4_tile_pack), the
// f16 pairs formed in shared memory (0.5625 bytes of W streamed per weight).
size_t q4_tile_bytes(int rows, int K);
int q4_tile_pack(cw_ctx* ctx, const void* payload, const void* scales, int rows, int K,
                 void* out);
int gemm_q4(cw_ctx* ctx, const void* xh, const void* xl, const void* wpack, int M, int N, int K,
            float* y, int ldy, const float* bias, int epi, float* ws = nullptr,
            size_t ws_bytes = 0, bool pdl = false);
// Packed Q4_0 [rows, K] -> wh, wl; X f32 [M, K] (row stride ldx) -> xh, xl.
int q4_split(cw_ctx* ctx, const void* payload, const void* scales, long rows, int K, void* wh,
             void* wl);
int x_split(cw_ctx* ctx, const float* x, long M, int K, int ldx, void* xh, void* xl);

}  // namespace cw
