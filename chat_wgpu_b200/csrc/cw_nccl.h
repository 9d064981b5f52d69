// cw_nccl.h -- the NCCL calls of the tensor-parallel decode (cw_nccl.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cw {

int tp_unique_id(uint8_t* id, size_t n);
int tp_comm_init(const uint8_t* id, int rank, int world, void** comm);
void tp_comm_destroy(void* comm);
// In-place all-reduces on `st` (graph-capturable).
int tp_sum_f32(void* comm, float* buf, size_t n, cudaStream_t st);
int tp_max_u64(void* comm, unsigned long long* buf, size_t n, cudaStream_t st);

}  // namespace cw
