// cw_noalloc.cu -- single-query attention for callers that cannot allocate
// device memory.
//
// Some hosts must not call cudaMalloc on the decode path: a runtime that owns
// every device allocation through its own pool, or a plugin inside a process
// whose allocator must never see a new block.  cw_attention (the op of
// attention.rs:7-38) needs scratch memory for its split-KV partial results
// and the per-kv-head counters that elect the CTA merging the splits, and
// takes both from the context's arena.  This entry point takes the same
// inputs and output as plain device pointers and keeps its scratch in one
// file-scope __device__ array instead, so it performs no allocation of any
// kind.
//
// The array (CW_NOALLOC_SCRATCH_BYTES, 1 MiB) lives in every GPU that loads
// the library until the process exits.  All calls on a device share it and it
// keeps the last call's contents: the counters are cleared by every call
// before its kernel, and two calls whose kernels overlap on the GPU (different
// streams, no ordering between them) race on it.  The array's device address
// is looked up once per device and kept for the life of the process, so the
// entry point must not be used on a device after cudaDeviceReset there.
#include <mutex>

#include "cw_common.h"
#include "cw_ops.h"

#define CW_NOALLOC_MAX_DEVICES 64

namespace cw {

// [0, 256): per-kv-head merge counters (64 x u32); [256, end): split partials.
static __device__ __align__(256) unsigned char g_attn_scratch[CW_NOALLOC_SCRATCH_BYTES];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[CW_NOALLOC_MAX_DEVICES];

// Device address of g_attn_scratch on `device`, looked up once per device
// with that device current.  In host code the symbol is only a host-side
// stand-in; kernels must receive this address.
static int scratch_address(int device, void** out) {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (!g_scratch_addr[device]) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p)
            return set_error(CW_ERR_CUDA, "cw_attention_noalloc: scratch address on device %d: %s",
                             device, cudaGetErrorString(e));
        g_scratch_addr[device] = p;
    }
    *out = g_scratch_addr[device];
    return CW_OK;
}

// Makes a device current for the length of one call and restores the
// thread's previous current device on destruction.
struct DeviceGuard {
    int prev = -1;
    cudaError_t enter(int device) {
        cudaError_t e = cudaGetDevice(&prev);
        if (e != cudaSuccess) {
            prev = -1;
            return e;
        }
        return prev == device ? cudaSuccess : cudaSetDevice(device);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace cw

using namespace cw;

extern "C" int cw_attention_noalloc(int device, void* stream, const float* q, const float* k,
                                    const float* v, float* out, size_t n_heads, size_t n_kv,
                                    size_t seq, size_t head_dim) {
    clear_error();
    CW_CHECK(q && k && v && out, CW_ERR_INVALID_ARG, "cw_attention_noalloc: NULL pointer argument");
    CW_CHECK(device >= 0 && device < CW_NOALLOC_MAX_DEVICES, CW_ERR_INVALID_ARG,
             "cw_attention_noalloc: device %d out of range", device);
    CW_CHECK(n_heads > 0 && n_kv > 0 && n_heads % n_kv == 0 && n_heads / n_kv <= 8,
             CW_ERR_INVALID_ARG,
             "cw_attention_noalloc: n_heads=%zu n_kv=%zu (need n_kv | n_heads, group <= 8)",
             n_heads, n_kv);
    CW_CHECK(n_kv <= 64, CW_ERR_INVALID_ARG, "cw_attention_noalloc: n_kv=%zu exceeds 64", n_kv);
    CW_CHECK(head_dim > 0 && head_dim <= 256, CW_ERR_INVALID_ARG,
             "cw_attention_noalloc: head_dim %zu (1..256)", head_dim);
    CW_CHECK(seq > 0 && seq < (1u << 30), CW_ERR_INVALID_ARG, "cw_attention_noalloc: seq must be >= 1");
    // the lookups below need `device` current; the caller's current device
    // is put back on every return path
    DeviceGuard guard;
    CW_CUDA(guard.enter(device));
    int sm = 0;
    CW_CUDA(cudaDeviceGetAttribute(&sm, cudaDevAttrMultiProcessorCount, device));
    // the same split count as cw_attention, so both give the same result
    const int n_splits = attention_splits_for(sm, (int)seq, (int)n_kv);
    const size_t part_bytes =
        n_splits > 1 ? n_heads * (size_t)n_splits * (head_dim + 2) * sizeof(float) : 0;
    CW_CHECK(part_bytes <= CW_NOALLOC_SCRATCH_BYTES - 256, CW_ERR_INVALID_ARG,
             "cw_attention_noalloc: %zu heads x %d splits x head_dim %zu need %zu bytes of "
             "scratch; the static scratch holds %d bytes (use cw_attention)",
             n_heads, n_splits, head_dim, part_bytes + 256, CW_NOALLOC_SCRATCH_BYTES);
    void* base = nullptr;
    CW_TRY(scratch_address(device, &base));
    unsigned* counters = reinterpret_cast<unsigned*>(base);
    float* part = reinterpret_cast<float*>(reinterpret_cast<unsigned char*>(base) + 256);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    CW_CUDA(cudaMemsetAsync(counters, 0, n_kv * sizeof(unsigned), st));
    return launch_attention_raw(st, q, k, v, out, (int)n_heads, (int)n_kv, (int)seq,
                                (int)head_dim, 0.0f, 0, (long)head_dim, (long)(n_kv * head_dim),
                                n_splits, part, counters);
}
