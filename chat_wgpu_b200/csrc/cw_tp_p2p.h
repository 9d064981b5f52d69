// cw_tp_p2p.h -- the tensor-parallel step's all-reduces over NVLink peer
// memory (cw_tp_p2p.cu).
#pragma once

#include <stdint.h>

#include "chatcuda.h"

namespace cw {

// One rank's exchange area and the peers' areas as mapped in this process.
struct TpP2P {
    void* mem = nullptr;  // this rank's area (cudaMalloc, exported by IPC handle)
    size_t bytes = 0;
    int rank = 0, world = 1, dim = 0;
    void* peer[CW_TP_MAX_WORLD] = {};  // every rank's area (this rank's: mem)
    void** d_peer = nullptr;            // the same table in device memory
    bool attached = false;
};

bool p2p_on(const cw_session* s);
int p2p_handle(cw_session* s, uint8_t* out);       // CW_TP_HANDLE_BYTES
int p2p_attach(cw_session* s, const uint8_t* blobs);  // world x CW_TP_HANDLE_BYTES
// In-place sum over the ranks of buf[dim] (all-reduce `idx` of the step).
int p2p_allreduce(cw_session* s, float* buf, int idx);
// The largest argmax key over the ranks into DevState::key.
int p2p_key(cw_session* s);
void p2p_free(cw_session* s);

}  // namespace cw
