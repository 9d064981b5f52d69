// mma_bench.cu -- latency and throughput of the warp-level integer MMA
// (mma.sync m16n8k32 u8 x u8 -> s32), the f16 MMA (m16n8k16) and dp4a on
// B200: the measurement behind the co-batched GEMV's choice of integer MMA
// products (csrc/cw_mgemv.cu).
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o /tmp/mma_bench \
//        chat_wgpu_b200/microbench/mma_bench.cu && /tmp/mma_bench
//
// Each kernel runs `iters` rounds of CH independent accumulation chains per
// warp (clock64 around the loop: cycles per round of one warp), first on one
// CTA, then on every SM (CUDA events: operations per second per SM).
#include <cstdio>
#include <cuda_runtime.h>
#include <cstdint>
template <int CH>
__global__ void k_imma(int iters, unsigned seed, long long* out, int* sink) {
    unsigned a[4] = {seed, seed * 3u, seed * 5u, seed * 7u};
    unsigned b0 = seed ^ 0x1234u, b1 = seed ^ 0x4321u;
    int d[CH][4];
    for (int c = 0; c < CH; c++) for (int e = 0; e < 4; e++) d[c][e] = c + e;
    __syncwarp();
    long long t0 = clock64();
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int c = 0; c < CH; c++)
            asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                         : "+r"(d[c][0]), "+r"(d[c][1]), "+r"(d[c][2]), "+r"(d[c][3])
                         : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
    long long t1 = clock64();
    int s = 0;
    for (int c = 0; c < CH; c++) for (int e = 0; e < 4; e++) s += d[c][e];
    sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
    if (threadIdx.x == 0) out[blockIdx.x * 32 + threadIdx.x / 32] = t1 - t0;
}
template <int CH>
__global__ void k_hmma(int iters, unsigned seed, long long* out, int* sink) {
    unsigned a[4] = {seed, seed * 3u, seed * 5u, seed * 7u};
    unsigned b0 = seed ^ 0x1234u, b1 = seed ^ 0x4321u;
    float d[CH][4];
    for (int c = 0; c < CH; c++) for (int e = 0; e < 4; e++) d[c][e] = 0.f;
    long long t0 = clock64();
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int c = 0; c < CH; c++)
            asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                         : "+f"(d[c][0]), "+f"(d[c][1]), "+f"(d[c][2]), "+f"(d[c][3])
                         : "r"(a[0] & 0x3c003c00u), "r"(a[1] & 0x3c003c00u), "r"(a[2] & 0x3c003c00u), "r"(a[3] & 0x3c003c00u), "r"(b0 & 0x3c003c00u), "r"(b1 & 0x3c003c00u));
    }
    long long t1 = clock64();
    float s = 0;
    for (int c = 0; c < CH; c++) for (int e = 0; e < 4; e++) s += d[c][e];
    sink[blockIdx.x * blockDim.x + threadIdx.x] = (int)s;
    if (threadIdx.x == 0) out[blockIdx.x * 32 + threadIdx.x / 32] = t1 - t0;
}
template <int CH>
__global__ void k_dp4a(int iters, unsigned seed, long long* out, int* sink) {
    int d[CH];
    for (int c = 0; c < CH; c++) d[c] = c;
    unsigned a = seed, b = seed * 3u;
    long long t0 = clock64();
    for (int i = 0; i < iters; i++) {
#pragma unroll
        for (int c = 0; c < CH; c++) asm volatile("dp4a.u32.u32 %0, %1, %2, %0;" : "+r"(d[c]) : "r"(a), "r"(b));
    }
    long long t1 = clock64();
    int s = 0;
    for (int c = 0; c < CH; c++) s += d[c];
    sink[blockIdx.x * blockDim.x + threadIdx.x] = s;
    if (threadIdx.x == 0) out[blockIdx.x * 32 + threadIdx.x / 32] = t1 - t0;
}
template <class F>
void run(const char* name, F kern, int warps, int iters, int ops_per_iter_per_warp) {
    long long* d_out; int* sink;
    cudaMalloc(&d_out, 32 * 8 * 148); cudaMalloc(&sink, 4 * 1024 * 148);
    kern<<<1, warps * 32>>>(iters, 7u, d_out, sink);
    cudaDeviceSynchronize();
    cudaEvent_t e0, e1; cudaEventCreate(&e0); cudaEventCreate(&e1);
    cudaEventRecord(e0);
    kern<<<148, warps * 32>>>(iters, 7u, d_out, sink);
    cudaEventRecord(e1);
    cudaError_t err = cudaDeviceSynchronize();
    float ms; cudaEventElapsedTime(&ms, e0, e1);
    long long cyc; cudaMemcpy(&cyc, d_out, 8, cudaMemcpyDeviceToHost);
    double per = (double)cyc / iters;
    printf("%-28s warps=%2d  cycles/iter=%8.2f  -> %.2f cycles per op per warp; grid time %.3f ms, %.3g ops/s/SM  [%s]\n",
           name, warps, per, per / ops_per_iter_per_warp, ms,
           (double)iters * ops_per_iter_per_warp * warps / (ms * 1e-3), cudaGetErrorString(err));
    cudaFree(d_out); cudaFree(sink);
}
int main() {
    const int it = 4096;
    run("imma chain x1", k_imma<1>, 1, it, 1);
    run("imma chains x4", k_imma<4>, 1, it, 4);
    run("imma chains x8", k_imma<8>, 1, it, 8);
    run("imma x4, 4 warps", k_imma<4>, 4, it, 4);
    run("imma x4, 16 warps", k_imma<4>, 16, it, 4);
    run("imma x8, 16 warps", k_imma<8>, 16, it, 8);
    run("hmma chain x1", k_hmma<1>, 1, it, 1);
    run("hmma chains x4", k_hmma<4>, 1, it, 4);
    run("hmma x4, 16 warps", k_hmma<4>, 16, it, 4);
    run("dp4a chains x8", k_dp4a<8>, 1, it, 8);
    run("dp4a x8, 16 warps", k_dp4a<8>, 16, it, 8);
    return 0;
}
