// cw_nccl.cu -- NCCL for the tensor-parallel decode (Qwen3-8B over 2-8 GPUs):
// the library is opened at run time (libnccl.so.2: the copy a PyTorch host has
// already loaded, else the system one), so libchatcuda.so keeps no link-time
// dependency on it and single-GPU hosts never need it.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "cw_common.h"
#include "cw_nccl.h"

namespace cw {

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t,
                               ncclComm_t, cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi& api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        a.get_unique_id = (decltype(a.get_unique_id))dlsym(h, "ncclGetUniqueId");
        a.comm_init_rank = (decltype(a.comm_init_rank))dlsym(h, "ncclCommInitRank");
        a.comm_destroy = (decltype(a.comm_destroy))dlsym(h, "ncclCommDestroy");
        a.all_reduce = (decltype(a.all_reduce))dlsym(h, "ncclAllReduce");
        a.error_string = (decltype(a.error_string))dlsym(h, "ncclGetErrorString");
        a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_reduce &&
               a.error_string;
    });
    return a;
}

int nccl_err(ncclResult_t r, const char* what) {
    return set_error(CW_ERR_CUDA, "%s: %s", what, api().error_string(r));
}

}  // namespace

int tp_unique_id(uint8_t* id, size_t n) {
    NcclApi& a = api();
    CW_CHECK(a.ok, CW_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    CW_CHECK(n >= sizeof(ncclUniqueId), CW_ERR_INVALID_ARG, "unique id buffer too small");
    ncclUniqueId u;
    ncclResult_t r = a.get_unique_id(&u);
    if (r != ncclSuccess) return nccl_err(r, "ncclGetUniqueId");
    memcpy(id, &u, sizeof u);
    return CW_OK;
}

int tp_comm_init(const uint8_t* id, int rank, int world, void** comm) {
    NcclApi& a = api();
    CW_CHECK(a.ok, CW_ERR_UNSUPPORTED, "libnccl.so.2 could not be loaded");
    ncclUniqueId u;
    memcpy(&u, id, sizeof u);
    ncclComm_t c = nullptr;
    ncclResult_t r = a.comm_init_rank(&c, world, u, rank);
    if (r != ncclSuccess) return nccl_err(r, "ncclCommInitRank");
    *comm = c;
    return CW_OK;
}

void tp_comm_destroy(void* comm) {
    if (comm && api().ok) api().comm_destroy((ncclComm_t)comm);
}

int tp_sum_f32(void* comm, float* buf, size_t n, cudaStream_t st) {
    ncclResult_t r = api().all_reduce(buf, buf, n, ncclFloat32, ncclSum, (ncclComm_t)comm, st);
    return r == ncclSuccess ? CW_OK : nccl_err(r, "ncclAllReduce(sum)");
}

int tp_max_u64(void* comm, unsigned long long* buf, size_t n, cudaStream_t st) {
    ncclResult_t r = api().all_reduce(buf, buf, n, ncclUint64, ncclMax, (ncclComm_t)comm, st);
    return r == ncclSuccess ? CW_OK : nccl_err(r, "ncclAllReduce(max)");
}

}  // namespace cw
