// cw_tp_p2p.cu -- the tensor-parallel decode's all-reduces over NVLink peer
// memory, in place of NCCL inside the per-stage step.
//
// Every rank of a session owns an exchange area (cudaMalloc'd, exported with
// a CUDA IPC handle and mapped by every other rank):
//   [0, 256)      argmax keys [2 parities][CW_TP_MAX_WORLD][2 halves] (u64 words)
//   [256, ...)    partial sums [2 parities][world][dim] (u64 words)
// Each u64 word carries a 32-bit payload and, in its high half, the epoch of
// the exchange that wrote it, so one aligned 8-byte store moves value and
// flag together: a reader knows a word has arrived when its epoch matches,
// with no fence or counter in between (the "low-latency" protocol of NCCL's
// LL kernels, restated).  All-reduce k of a session (the O and down partial
// sums of each layer, in order) has epoch k + 1 and parity k % 2: thread i of
// every rank stores element i of its partial to slot [k % 2][rank] of every
// peer (plain 8-byte NVLink stores), then reads element i of every rank's slot
// in its own area, waiting (bounded) for each to show the epoch, and sums the
// world values in rank order -- the same order, hence the same bits, on every
// rank.  Two parities suffice: a rank reaches exchange k + 2 only after every
// rank has pushed k + 1, which each does after it finished reading k.
// k comes from DevState::ar_seq (advanced by the step's finalize kernel) plus
// the all-reduce's index within the step; the LM head's argmax key goes the
// same way (two words, DevState::key_seq).  A wait that runs out (P2P_WAIT_NS)
// reports DEV_TIMEOUT, which the host turns into CW_ERR_TIMEOUT.  No TMA, no
// multicast, no library kernel on peer memory: plain loads and stores.
#include <string.h>

#include <memory>
#include <utility>
#include <vector>

#include "cw_common.h"
#include "cw_device.cuh"
#include "cw_gemv.cuh"
#include "cw_model.h"
#include "cw_tp_p2p.h"

namespace cw {

namespace {

constexpr int P2P_THREADS = 128;
constexpr size_t P2P_RECV_OFF = 256;
constexpr uint64_t P2P_WAIT_NS = 2000000000ull;  // 2 s
constexpr uint32_t P2P_MAGIC = 0x32505743u;      // "CWP2"

struct Blob {  // what one rank hands the others (CW_TP_HANDLE_BYTES)
    cudaIpcMemHandle_t ipc;  // 64 bytes
    uint8_t uuid[16];        // the GPU, so that no two ranks share one
    int32_t rank, world, dim;
    uint32_t magic;
    uint8_t pad[CW_TP_HANDLE_BYTES - 64 - 16 - 16];
};
static_assert(sizeof(Blob) == CW_TP_HANDLE_BYTES, "handle blob size");

__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned long long ll_word(unsigned payload, unsigned epoch) {
    return ((unsigned long long)epoch << 32) | payload;
}
// Bounded wait (this thread) for the word at p to carry `epoch`; its payload.
__device__ __forceinline__ bool ll_read(const unsigned long long* p, unsigned epoch,
                                        unsigned* payload) {
    unsigned long long w = ld_relaxed_sys_u64(p);
    if ((unsigned)(w >> 32) != epoch) {
        const uint64_t t0 = global_ns();
        do {
            if (global_ns() - t0 > P2P_WAIT_NS) return false;
            w = ld_relaxed_sys_u64(p);
        } while ((unsigned)(w >> 32) != epoch);
    }
    *payload = (unsigned)w;
    return true;
}

__global__ void __launch_bounds__(P2P_THREADS)
    k_p2p_allreduce(float* buf, int dim, const DevState* st, void* const* peers, int rank,
                    int world, int idx, int* status) {
    pdl_trigger();
    pdl_wait();  // the partial sums in buf are complete
    const unsigned k = st->ar_seq + (unsigned)idx, epoch = k + 1u;
    const size_t par = k & 1u;
    const int i = blockIdx.x * P2P_THREADS + threadIdx.x;
    if (i >= dim) return;
    const float v = buf[i];
    const unsigned long long w = ll_word(__float_as_uint(v), epoch);
    for (int r = 0; r < world; r++)
        if (r != rank)
            st_relaxed_sys_u64(reinterpret_cast<unsigned long long*>(
                                   static_cast<char*>(peers[r]) + P2P_RECV_OFF) +
                                   (par * world + rank) * dim + i,
                               w);
    const unsigned long long* own =
        reinterpret_cast<const unsigned long long*>(static_cast<const char*>(peers[rank]) +
                                                    P2P_RECV_OFF) +
        par * world * dim + i;
    float sum = 0.f;
    for (int r = 0; r < world; r++) {  // rank order
        unsigned x = __float_as_uint(v);
        if (r != rank && !ll_read(own + (size_t)r * dim, epoch, &x)) {
            atomicCAS(status, (int)DEV_OK, (int)DEV_TIMEOUT);
            return;
        }
        sum += __uint_as_float(x);
    }
    buf[i] = sum;
}

// The argmax key over the ranks' vocabulary shards: every rank's st->key
// (this step's best (logit, index) on its shard) to every rank as two words,
// the largest kept.  One thread.
__global__ void k_p2p_key(DevState* st, void* const* peers, int rank, int world, int* status) {
    pdl_trigger();
    pdl_wait();
    const unsigned k = st->key_seq, epoch = k + 1u;
    const size_t par = k & 1u;
    const unsigned long long mine = st->key;
    for (int r = 0; r < world; r++) {
        if (r == rank) continue;
        unsigned long long* slot = static_cast<unsigned long long*>(peers[r]) +
                                   (par * CW_TP_MAX_WORLD + rank) * 2;
        st_relaxed_sys_u64(slot, ll_word((unsigned)mine, epoch));
        st_relaxed_sys_u64(slot + 1, ll_word((unsigned)(mine >> 32), epoch));
    }
    const unsigned long long* own =
        static_cast<const unsigned long long*>(peers[rank]) + par * CW_TP_MAX_WORLD * 2;
    unsigned long long best = mine;
    for (int r = 0; r < world; r++) {
        if (r == rank) continue;
        unsigned lo, hi;
        if (!ll_read(own + 2 * r, epoch, &lo) || !ll_read(own + 2 * r + 1, epoch, &hi)) {
            atomicCAS(status, (int)DEV_OK, (int)DEV_TIMEOUT);
            return;
        }
        const unsigned long long kk = ((unsigned long long)hi << 32) | lo;
        best = kk > best ? kk : best;
    }
    st->key = best;
    st->key_seq = k + 1u;
}

template <typename... KArgs, typename... Args>
int p2p_launch(cw_ctx* ctx, void (*kern)(KArgs...), dim3 grid, dim3 block, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = ctx->pdl ? 1 : 0;
    CW_CUDA(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
    return check_launch("tensor-parallel all-reduce");
}

int device_uuid(int device, uint8_t* out) {
    cudaDeviceProp prop{};
    CW_CUDA(cudaGetDeviceProperties(&prop, device));
    memcpy(out, &prop.uuid, 16);
    return CW_OK;
}

}  // namespace

bool p2p_on(const cw_session* s) {
    return s->p2p && static_cast<const TpP2P*>(s->p2p)->attached;
}

int p2p_handle(cw_session* s, uint8_t* out) {
    cw_model* m = s->m;
    CW_CHECK(m->tp_world > 1, CW_ERR_UNSUPPORTED,
             "cw_session_tp_handle: the model is not tensor-parallel");
    CW_CHECK(m->tp_world <= CW_TP_MAX_WORLD, CW_ERR_UNSUPPORTED,
             "cw_session_tp_handle: world %d > %d", m->tp_world, CW_TP_MAX_WORLD);
    const int dim = (int)m->info.dim;
    if (!s->p2p) {
        std::unique_ptr<TpP2P> p(new TpP2P());
        p->rank = m->tp_rank;
        p->world = m->tp_world;
        p->dim = dim;
        p->bytes = P2P_RECV_OFF + (size_t)2 * p->world * dim * sizeof(unsigned long long);
        CW_CUDA(cudaMalloc(&p->mem, p->bytes));
        cudaError_t e = cudaMemset(p->mem, 0, p->bytes);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess) {
            cudaFree(p->mem);
            return set_error(CW_ERR_CUDA, "tensor-parallel exchange area: %s", cudaGetErrorString(e));
        }
        s->p2p = p.release();
    }
    TpP2P* p = static_cast<TpP2P*>(s->p2p);
    Blob b;
    memset(&b, 0, sizeof b);
    CW_CUDA(cudaIpcGetMemHandle(&b.ipc, p->mem));
    CW_TRY(device_uuid(s->ctx->device, b.uuid));
    b.rank = p->rank;
    b.world = p->world;
    b.dim = p->dim;
    b.magic = P2P_MAGIC;
    memcpy(out, &b, sizeof b);
    return CW_OK;
}

int p2p_attach(cw_session* s, const uint8_t* blobs) {
    CW_CHECK(s->p2p, CW_ERR_INVALID_ARG, "cw_session_tp_attach: call cw_session_tp_handle first");
    TpP2P* p = static_cast<TpP2P*>(s->p2p);
    CW_CHECK(!p->attached, CW_ERR_INVALID_ARG, "cw_session_tp_attach: already attached");
    std::vector<Blob> b((size_t)p->world);
    memcpy(b.data(), blobs, (size_t)p->world * sizeof(Blob));
    for (int r = 0; r < p->world; r++) {
        CW_CHECK(b[r].magic == P2P_MAGIC && b[r].rank == r && b[r].world == p->world &&
                     b[r].dim == p->dim,
                 CW_ERR_INVALID_ARG, "cw_session_tp_attach: handle %d is not rank %d of %d", r, r,
                 p->world);
        for (int q = 0; q < r; q++)
            CW_CHECK(memcmp(b[q].uuid, b[r].uuid, 16) != 0, CW_ERR_UNSUPPORTED,
                     "cw_session_tp_attach: ranks %d and %d are on the same GPU", q, r);
    }
    uint8_t mine[16];
    CW_TRY(device_uuid(s->ctx->device, mine));
    CW_CHECK(memcmp(mine, b[p->rank].uuid, 16) == 0, CW_ERR_INVALID_ARG,
             "cw_session_tp_attach: handle %d is not this session's", p->rank);
    int rc = CW_OK;
    for (int r = 0; r < p->world && rc == CW_OK; r++) {
        if (r == p->rank) {
            p->peer[r] = p->mem;
            continue;
        }
        cudaError_t e = cudaIpcOpenMemHandle(&p->peer[r], b[r].ipc, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            p->peer[r] = nullptr;
            rc = set_error(CW_ERR_CUDA, "cw_session_tp_attach: mapping rank %d: %s", r,
                           cudaGetErrorString(e));
        }
    }
    if (rc == CW_OK) {
        cudaError_t e = cudaMalloc(&p->d_peer, sizeof(void*) * CW_TP_MAX_WORLD);
        if (e == cudaSuccess)
            e = cudaMemcpy(p->d_peer, p->peer, sizeof(void*) * CW_TP_MAX_WORLD,
                           cudaMemcpyHostToDevice);
        // the exchange sequence starts over (every word of every area is still
        // at epoch 0, which no exchange uses)
        if (e == cudaSuccess) e = cudaMemset(&s->st->ar_seq, 0, sizeof(unsigned));
        if (e == cudaSuccess) e = cudaMemset(&s->st->key_seq, 0, sizeof(unsigned));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess)
            rc = set_error(CW_ERR_CUDA, "cw_session_tp_attach: %s", cudaGetErrorString(e));
    }
    if (rc != CW_OK) {
        for (int r = 0; r < p->world; r++)
            if (r != p->rank && p->peer[r]) cudaIpcCloseMemHandle(p->peer[r]);
        memset(p->peer, 0, sizeof p->peer);
        if (p->d_peer) cudaFree(p->d_peer);
        p->d_peer = nullptr;
        return rc;
    }
    p->attached = true;
    return CW_OK;
}

int p2p_allreduce(cw_session* s, float* buf, int idx) {
    TpP2P* p = static_cast<TpP2P*>(s->p2p);
    const int blocks = (p->dim + P2P_THREADS - 1) / P2P_THREADS;
    return p2p_launch(s->ctx, k_p2p_allreduce, dim3(blocks), dim3(P2P_THREADS), buf, p->dim,
                      (const DevState*)s->st, (void* const*)p->d_peer, p->rank, p->world, idx,
                      s->ctx->d_status);
}

int p2p_key(cw_session* s) {
    TpP2P* p = static_cast<TpP2P*>(s->p2p);
    return p2p_launch(s->ctx, k_p2p_key, dim3(1), dim3(1), s->st, (void* const*)p->d_peer,
                      p->rank, p->world, s->ctx->d_status);
}

void p2p_free(cw_session* s) {
    TpP2P* p = static_cast<TpP2P*>(s->p2p);
    if (!p) return;
    for (int r = 0; r < p->world; r++)
        if (r != p->rank && p->peer[r]) cudaIpcCloseMemHandle(p->peer[r]);
    if (p->d_peer) cudaFree(p->d_peer);
    if (p->mem) cudaFree(p->mem);
    delete p;
    s->p2p = nullptr;
}

}  // namespace cw
