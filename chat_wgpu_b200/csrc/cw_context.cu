// cw_context.cu -- the GpuContext replacement (chat-wgpu src/context.rs):
// device + stream, buffer table, per-frame arena, copy/read, CUDA-event
// profiler, errors.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <cmath>

#include "cw_common.h"

namespace cw {

static thread_local std::string g_err;

int set_error(int status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    return status;
}

// Clears this thread's message and any non-sticky CUDA error left by an
// earlier call, so a later launch check reports only its own failure.
void clear_error() {
    g_err.clear();
    (void)cudaGetLastError();
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return set_error(CW_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return CW_OK;
}

int buf_get(cw_ctx* ctx, cw_buf b, BufEntry** out, size_t min_bytes, const char* what) {
    auto it = ctx->bufs.find(b);
    if (b == 0 || it == ctx->bufs.end())
        return set_error(CW_ERR_INVALID_ARG, "%s: invalid buffer handle %llu", what,
                         (unsigned long long)b);
    if (it->second.nbytes < min_bytes)
        return set_error(CW_ERR_INVALID_ARG, "%s: buffer %llu holds %zu bytes, need %zu", what,
                         (unsigned long long)b, it->second.nbytes, min_bytes);
    *out = &it->second;
    return CW_OK;
}

int buf_new(cw_ctx* ctx, size_t nbytes, int kind, cw_buf* out, BufEntry** entry) {
    void* p = nullptr;
    // Round up so vector loads past a ragged tail stay inside the allocation.
    size_t alloc = (std::max<size_t>(nbytes, 1) + 255) & ~size_t(255);
    CW_CUDA(cudaMalloc(&p, alloc));
    uint64_t id = ctx->next_id++;
    BufEntry e;
    e.ptr = p;
    e.nbytes = nbytes;
    e.kind = kind;
    ctx->bufs[id] = e;
    *out = id;
    if (entry) *entry = &ctx->bufs[id];
    return CW_OK;
}

// context.rs:207-227: slot `cursor` is reused while its size is unchanged,
// reallocated otherwise.
int arena_get(cw_ctx* ctx, size_t len, cw_buf* out, BufEntry** entry) {
    size_t c = ctx->cursor++;
    if (c < ctx->arena.size()) {
        auto& slot = ctx->arena[c];
        if (slot.first == len) {
            *out = slot.second;
            if (entry) *entry = &ctx->bufs[slot.second];
            return CW_OK;
        }
        // size changed: free the old slot buffer (stream-ordered after prior use)
        auto it = ctx->bufs.find(slot.second);
        if (it != ctx->bufs.end()) {
            CW_CUDA(cudaStreamSynchronize(ctx->stream));
            cudaFree(it->second.ptr);
            ctx->bufs.erase(it);
        }
        cw_buf b;
        CW_TRY(buf_new(ctx, len * 4, BUF_ARENA, &b, entry));
        slot = {len, b};
        *out = b;
        return CW_OK;
    }
    cw_buf b;
    CW_TRY(buf_new(ctx, len * 4, BUF_ARENA, &b, entry));
    ctx->arena.push_back({len, b});
    *out = b;
    return CW_OK;
}

int check_device_status(cw_ctx* ctx) {
    int st = 0;
    CW_CUDA(cudaMemcpyAsync(&st, ctx->d_status, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream));
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    if (st != DEV_OK) {
        int zero = 0;
        cudaMemcpyAsync(ctx->d_status, &zero, sizeof(int), cudaMemcpyHostToDevice, ctx->stream);
        cudaStreamSynchronize(ctx->stream);
        if (st == DEV_TIMEOUT)
            return set_error(CW_ERR_TIMEOUT, "a bounded device-side wait timed out");
        return set_error(CW_ERR_INVALID_ARG, "device kernel rejected its input (status %d)", st);
    }
    return CW_OK;
}

OpScope::OpScope(cw_ctx* c, const char* n) : ctx(c), name(n) {
    if (!ctx->profiling) return;
    auto take = [&]() {
        cudaEvent_t e;
        if (!ctx->event_pool.empty()) {
            e = ctx->event_pool.back();
            ctx->event_pool.pop_back();
        } else {
            cudaEventCreate(&e);
        }
        return e;
    };
    start = take();
    stop = take();
    // Inside stream capture a plain record only tracks dependencies; the
    // External flag makes it an event-record node that timestamps on replay.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(ctx->stream, &cs);
    flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : 0;
    cudaEventRecordWithFlags(start, ctx->stream, flags);
}

OpScope::~OpScope() {
    if (!start) return;
    cudaEventRecordWithFlags(stop, ctx->stream, flags);
    ctx->prof.push_back({name, start, stop});
}

int ensure_counters(cw_ctx* ctx, size_t n) {
    if (n <= ctx->n_counters) return CW_OK;
    size_t m = std::max<size_t>(n, 256);
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    if (ctx->d_counters) cudaFree(ctx->d_counters);
    ctx->d_counters = nullptr;
    ctx->n_counters = 0;
    CW_CUDA(cudaMalloc(&ctx->d_counters, m * sizeof(unsigned)));
    // on the context stream: kernels there do not wait for the legacy stream
    CW_CUDA(cudaMemsetAsync(ctx->d_counters, 0, m * sizeof(unsigned), ctx->stream));
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    ctx->n_counters = m;
    return CW_OK;
}

int rope_table(cw_ctx* ctx, uint32_t head_dim, float theta, const float** out) {
    uint32_t tb;
    memcpy(&tb, &theta, 4);
    auto key = std::make_pair(head_dim, tb);
    auto it = ctx->rope_tables.find(key);
    if (it != ctx->rope_tables.end()) {
        *out = it->second;
        return CW_OK;
    }
    uint32_t half = head_dim / 2;
    std::vector<float> t(std::max<uint32_t>(half, 1));
    for (uint32_t i = 0; i < half; i++) {
        // rope.wgsl:26-27: exponent = -2.0 * f32(i) / f32(head_dim); pow(theta, exponent)
        float exponent = -2.0f * (float)i / (float)head_dim;
        t[i] = powf(theta, exponent);
    }
    float* d = nullptr;
    CW_CUDA(cudaMalloc(&d, t.size() * sizeof(float)));
    // on the context stream (the non-blocking stream does not wait for the
    // legacy default stream a plain cudaMemcpy uses), complete before t dies
    CW_CUDA(cudaMemcpyAsync(d, t.data(), t.size() * sizeof(float), cudaMemcpyHostToDevice,
                            ctx->stream));
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    ctx->rope_tables[key] = d;
    *out = d;
    return CW_OK;
}

}  // namespace cw

using namespace cw;

extern "C" {

const char* cw_last_error(void) { return g_err.c_str(); }

int cw_abi_version(void) { return CW_ABI_VERSION; }

int cw_ctx_create(int device, cw_ctx** out) {
    clear_error();
    CW_CHECK(out, CW_ERR_INVALID_ARG, "cw_ctx_create: out is NULL");
    *out = nullptr;
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0)
        return set_error(CW_ERR_NO_DEVICE, "no CUDA device: %s", cudaGetErrorString(e));
    CW_CHECK(device >= 0 && device < n, CW_ERR_NO_DEVICE, "device %d out of range (%d devices)",
             device, n);
    cudaDeviceProp prop;
    CW_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10 || prop.minor != 0)
        return set_error(CW_ERR_NO_DEVICE,
                         "device %d is sm_%d%d; libchatcuda.so is built for sm_100a only", device,
                         prop.major, prop.minor);
    CW_CUDA(cudaSetDevice(device));
    cw_ctx* c = new cw_ctx();
    c->device = device;
    c->sm_count = prop.multiProcessorCount;
    cudaDeviceGetAttribute(&c->clock_khz, cudaDevAttrClockRate, c->device);
    if (c->clock_khz <= 0) c->clock_khz = 1;
    c->l2_bytes = prop.l2CacheSize;
    c->max_smem_optin = (int)prop.sharedMemPerBlockOptin;
    c->smem_per_sm = (int)prop.sharedMemPerMultiprocessor;
    char b[320];
    snprintf(b, sizeof b, "CUDA sm_%d%da (%s)", prop.major, prop.minor, prop.name);
    c->backend = b;
    cudaError_t e1 = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
    cudaError_t e2 = cudaMalloc(&c->d_status, sizeof(int));
    if (e1 != cudaSuccess || e2 != cudaSuccess) {
        delete c;
        return set_error(CW_ERR_CUDA, "context setup failed: %s",
                         cudaGetErrorString(e1 != cudaSuccess ? e1 : e2));
    }
    cudaMemsetAsync(c->d_status, 0, sizeof(int), c->stream);  // ordered with c's kernels
    int rc = ensure_counters(c, 1024);
    if (rc != CW_OK) {
        cw_ctx_destroy(c);
        return rc;
    }
    *out = c;
    return CW_OK;
}

int cw_ctx_destroy(cw_ctx* ctx) {
    if (!ctx) return CW_OK;
    cudaSetDevice(ctx->device);
    if (ctx->stream) cudaStreamSynchronize(ctx->stream);
    for (auto& kv : ctx->bufs) cudaFree(kv.second.ptr);
    for (auto& kv : ctx->rope_tables) cudaFree(kv.second);
    for (auto& p : ctx->prof) {
        cudaEventDestroy(p.start);
        cudaEventDestroy(p.stop);
    }
    for (auto e : ctx->event_pool) cudaEventDestroy(e);
    if (ctx->d_status) cudaFree(ctx->d_status);
    if (ctx->d_counters) cudaFree(ctx->d_counters);
    if (ctx->gemm_scratch) cudaFree(ctx->gemm_scratch);
    if (ctx->stream) cudaStreamDestroy(ctx->stream);
    delete ctx;
    return CW_OK;
}

int cw_ctx_backend(cw_ctx* ctx, char* buf, size_t cap) {
    CW_CHECK(ctx && buf && cap, CW_ERR_INVALID_ARG, "cw_ctx_backend: bad arguments");
    snprintf(buf, cap, "%s", ctx->backend.c_str());
    return CW_OK;
}

int cw_ctx_device(cw_ctx* ctx, int* device) {
    CW_CHECK(ctx && device, CW_ERR_INVALID_ARG, "cw_ctx_device: bad arguments");
    *device = ctx->device;
    return CW_OK;
}

int cw_ctx_set_pdl(cw_ctx* ctx, int on) {
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_ctx_set_pdl: ctx is NULL");
    ctx->pdl = on != 0;
    return CW_OK;
}

int cw_ctx_stream(cw_ctx* ctx, void** stream) {
    CW_CHECK(ctx && stream, CW_ERR_INVALID_ARG, "cw_ctx_stream: bad arguments");
    *stream = (void*)ctx->stream;
    return CW_OK;
}

static int upload(cw_ctx* ctx, const void* data, size_t nbytes, cw_buf* out) {
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "upload: bad arguments");
    CW_CHECK(data || nbytes == 0, CW_ERR_INVALID_ARG, "upload: data is NULL");
    cudaSetDevice(ctx->device);
    BufEntry* e;
    CW_TRY(buf_new(ctx, nbytes, BUF_STORAGE, out, &e));
    if (nbytes) {
        CW_CUDA(cudaMemcpyAsync(e->ptr, data, nbytes, cudaMemcpyHostToDevice, ctx->stream));
        CW_CUDA(cudaStreamSynchronize(ctx->stream));  // caller may free `data`
    }
    return CW_OK;
}

int cw_storage(cw_ctx* ctx, const float* data, size_t len, cw_buf* out) {
    clear_error();
    return upload(ctx, data, len * 4, out);
}

int cw_storage_u32(cw_ctx* ctx, const uint32_t* data, size_t len, cw_buf* out) {
    clear_error();
    return upload(ctx, data, len * 4, out);
}

int cw_storage_bytes(cw_ctx* ctx, const void* data, size_t nbytes, cw_buf* out) {
    clear_error();
    return upload(ctx, data, nbytes, out);
}

int cw_empty(cw_ctx* ctx, size_t len, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_empty: bad arguments");
    cudaSetDevice(ctx->device);
    return arena_get(ctx, len, out);
}

int cw_empty_persistent(cw_ctx* ctx, size_t len, cw_buf* out) {
    clear_error();
    CW_CHECK(ctx && out, CW_ERR_INVALID_ARG, "cw_empty_persistent: bad arguments");
    cudaSetDevice(ctx->device);
    BufEntry* e;
    CW_TRY(buf_new(ctx, len * 4, BUF_PERSISTENT, out, &e));
    CW_CUDA(cudaMemsetAsync(e->ptr, 0, len * 4, ctx->stream));
    return CW_OK;
}

int cw_buf_release(cw_ctx* ctx, cw_buf buf) {
    clear_error();
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_buf_release: ctx is NULL");
    BufEntry* e;
    CW_TRY(buf_get(ctx, buf, &e, 0, "cw_buf_release"));
    CW_CHECK(e->kind != BUF_ARENA, CW_ERR_INVALID_ARG,
             "cw_buf_release: arena buffers belong to the context");
    cudaSetDevice(ctx->device);
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    cudaFree(e->ptr);
    ctx->bufs.erase(buf);
    return CW_OK;
}

int cw_buf_nbytes(cw_ctx* ctx, cw_buf buf, size_t* nbytes) {
    clear_error();
    CW_CHECK(ctx && nbytes, CW_ERR_INVALID_ARG, "cw_buf_nbytes: bad arguments");
    BufEntry* e;
    CW_TRY(buf_get(ctx, buf, &e, 0, "cw_buf_nbytes"));
    *nbytes = e->nbytes;
    return CW_OK;
}

int cw_buf_device_ptr(cw_ctx* ctx, cw_buf buf, void** dptr) {
    clear_error();
    CW_CHECK(ctx && dptr, CW_ERR_INVALID_ARG, "cw_buf_device_ptr: bad arguments");
    BufEntry* e;
    CW_TRY(buf_get(ctx, buf, &e, 0, "cw_buf_device_ptr"));
    *dptr = e->ptr;
    return CW_OK;
}

int cw_copy(cw_ctx* ctx, cw_buf src, size_t src_off, cw_buf dst, size_t dst_off, size_t len) {
    clear_error();
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_copy: ctx is NULL");
    BufEntry *s, *d;
    CW_TRY(buf_get(ctx, src, &s, (src_off + len) * 4, "cw_copy(src)"));
    CW_TRY(buf_get(ctx, dst, &d, (dst_off + len) * 4, "cw_copy(dst)"));
    if (!len) return CW_OK;
    cudaSetDevice(ctx->device);
    OpScope scope(ctx, "copy");
    CW_CUDA(cudaMemcpyAsync((char*)d->ptr + dst_off * 4, (const char*)s->ptr + src_off * 4,
                            len * 4, cudaMemcpyDeviceToDevice, ctx->stream));
    return CW_OK;
}

int cw_write(cw_ctx* ctx, cw_buf dst, size_t dst_off, const float* data, size_t len) {
    clear_error();
    CW_CHECK(ctx && (data || !len), CW_ERR_INVALID_ARG, "cw_write: bad arguments");
    BufEntry* d;
    CW_TRY(buf_get(ctx, dst, &d, (dst_off + len) * 4, "cw_write"));
    if (!len) return CW_OK;
    cudaSetDevice(ctx->device);
    CW_CUDA(cudaMemcpyAsync((char*)d->ptr + dst_off * 4, data, len * 4, cudaMemcpyHostToDevice,
                            ctx->stream));
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    return CW_OK;
}

static int read_bytes(cw_ctx* ctx, cw_buf src, void* out, size_t nbytes, const char* what) {
    clear_error();
    CW_CHECK(ctx && (out || !nbytes), CW_ERR_INVALID_ARG, "%s: bad arguments", what);
    BufEntry* s;
    CW_TRY(buf_get(ctx, src, &s, nbytes, what));
    cudaSetDevice(ctx->device);
    CW_TRY(check_launch(what));
    if (nbytes)
        CW_CUDA(cudaMemcpyAsync(out, s->ptr, nbytes, cudaMemcpyDeviceToHost, ctx->stream));
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    return check_device_status(ctx);
}

int cw_read(cw_ctx* ctx, cw_buf src, float* out, size_t len) {
    return read_bytes(ctx, src, out, len * 4, "cw_read");
}

int cw_read_u32(cw_ctx* ctx, cw_buf src, uint32_t* out, size_t len) {
    return read_bytes(ctx, src, out, len * 4, "cw_read_u32");
}

int cw_flush(cw_ctx* ctx) {
    clear_error();
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_flush: ctx is NULL");
    return check_launch("cw_flush");
}

int cw_sync(cw_ctx* ctx) {
    clear_error();
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_sync: ctx is NULL");
    cudaSetDevice(ctx->device);
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    return check_device_status(ctx);
}

int cw_reset_frame(cw_ctx* ctx) {
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_reset_frame: ctx is NULL");
    ctx->cursor = 0;
    return CW_OK;
}

int cw_clear_cache(cw_ctx* ctx) {
    clear_error();
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_clear_cache: ctx is NULL");
    cudaSetDevice(ctx->device);
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    for (auto& slot : ctx->arena) {
        auto it = ctx->bufs.find(slot.second);
        if (it != ctx->bufs.end()) {
            cudaFree(it->second.ptr);
            ctx->bufs.erase(it);
        }
    }
    ctx->arena.clear();
    ctx->cursor = 0;
    return CW_OK;
}

int cw_begin_profile(cw_ctx* ctx) {
    clear_error();
    CW_CHECK(ctx, CW_ERR_INVALID_ARG, "cw_begin_profile: ctx is NULL");
    for (auto& p : ctx->prof) {
        ctx->event_pool.push_back(p.start);
        ctx->event_pool.push_back(p.stop);
    }
    ctx->prof.clear();
    ctx->profiling = true;
    return CW_OK;
}

int cw_report_profile(cw_ctx* ctx, cw_profile_row* rows, size_t cap, size_t* n_rows) {
    clear_error();
    CW_CHECK(ctx && n_rows, CW_ERR_INVALID_ARG, "cw_report_profile: bad arguments");
    cudaSetDevice(ctx->device);
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    std::map<std::string, std::pair<uint32_t, double>> agg;
    for (auto& p : ctx->prof) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, p.start, p.stop);
        auto& a = agg[p.name];
        a.first += 1;
        a.second += ms;
        ctx->event_pool.push_back(p.start);
        ctx->event_pool.push_back(p.stop);
    }
    ctx->prof.clear();
    ctx->profiling = false;
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

}  // extern "C"
