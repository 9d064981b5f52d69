// ring_bench.cu -- how fast one CTA per SM can stream HBM into shared memory
// through a ring of cp.async.bulk copies, and what the consumer side costs.
// The measurement behind the weight rings of the persistent decode step
// (csrc/cw_step.cuh) and the co-batched GEMV (csrc/cw_mgemv.cu).
//
//   nvcc -gencode arch=compute_100a,code=sm_100a -O3 -o /tmp/ring_bench \
//        chat_wgpu_b200/microbench/ring_bench.cu && /tmp/ring_bench
//
// A 4 GiB buffer is split over 148 x (CTAs per SM) CTAs; in each, lane 0 of
// warp 0 copies its range slot by slot into a ring of S stages (one bulk copy
// per slot, L2 evict-first or evict-normal), refilling a stage once its
// "empty" mbarrier completes.  Consumer modes:
//   0  one thread waits for each slot and releases it
//   1  16 warps wait, named barrier, one thread releases
//   2  16 warps wait, each warp's lane 0 releases (16 arrivals per slot)
//   3  mode 1, every thread also reading its share of the slot
//   4  mode 2, with the reads
//   5  mode 3, plus `work` dependent FMAs per 16 bytes read
//   6  mode 5 with the 16 warps in two groups of 8 taking alternate slots,
//      each group with its own named barrier
// Every wait is bounded; on a timeout the kernel records it in `err` and the
// producer waits (bounded) for its copies in flight before the CTA exits.
#include <cstdint>
#include <cstdio>

#include <cuda_runtime.h>

__device__ __forceinline__ uint32_t sa(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ bool try_wait(uint64_t* b, unsigned par) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0,1,0,p;\n\t}"
        : "=r"(ok)
        : "r"(sa(b)), "r"(par)
        : "memory");
    return ok;
}
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// bounded wait (1 s)
__device__ __forceinline__ bool wait_phase(uint64_t* b, unsigned par) {
    if (try_wait(b, par)) return true;
    const uint64_t t0 = now_ns();
    while (!try_wait(b, par))
        if (now_ns() - t0 > 1000000000ull) return false;
    return true;
}
// named barrier `id` over `n` consumer threads (the producer warp never
// joins); returns whether any of them passed v != 0
__device__ __forceinline__ bool group_sync_or(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(b)) : "memory");
}

__global__ void k_ring(const uint8_t* src, size_t per_cta, int S, int slot, int* err,
                       int evict_first, int mode, int work) {
    extern __shared__ __align__(128) uint8_t sm[];
    __shared__ uint64_t full[32], empty[32];
    __shared__ volatile int stop;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        const int cnt = (mode == 2 || mode == 4) ? 16 : 1;
        for (int i = 0; i < S; i++) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&full[i])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sa(&empty[i])), "r"(cnt));
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        stop = 0;
    }
    __syncthreads();
    const int n = (int)(per_cta / slot);
    const uint8_t* base = src + (size_t)blockIdx.x * per_cta;
    if (warp == 0) {  // the producer
        if (lane != 0) return;
        uint64_t pol;
        if (evict_first)
            asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
        else
            asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
        int q = 0;
        for (; q < n && !stop; q++) {
            const int st = q % S;
            if (q >= S && !wait_phase(&empty[st], ((q / S) - 1) & 1)) {
                atomicExch(err, 1);
                stop = 1;
                break;
            }
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(&full[st])),
                         "r"(slot)
                         : "memory");
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
                " [%0], [%1], %2, [%3], %4;" ::"r"(sa(sm + (size_t)st * slot)),
                "l"(base + (size_t)q * slot), "r"(slot), "r"(sa(&full[st])), "l"(pol)
                : "memory");
        }
        // the last (at most S) copies may still be landing: wait for them
        for (int k = q - S < 0 ? 0 : q - S; k < q; k++) wait_phase(&full[k % S], (k / S) & 1);
        return;
    }
    const int cw = warp - 1;  // consumer warp 0..15
    if (mode == 0) {
        if (cw == 0 && lane == 0) {
            for (int q = 0; q < n && !stop; q++) {
                const int st = q % S;
                if (!wait_phase(&full[st], (q / S) & 1)) {
                    atomicExch(err, 2);
                    stop = 1;
                    break;
                }
                arrive(&empty[st]);
            }
        }
        return;
    }
    unsigned acc = 0;
    float facc = 0.f;
    const int grp = mode == 6 ? (cw >= 8) : 0;
    const int gthreads = mode == 6 ? 256 : 512;
    for (int q = grp; q < n; q += (mode == 6 ? 2 : 1)) {
        const int st = q % S;
        bool ok = wait_phase(&full[st], (q / S) & 1);
        if (ok && mode >= 3) {
            const uint4* p = reinterpret_cast<const uint4*>(sm + (size_t)st * slot);
            const int nv = slot / 16;
            const int t0 = mode == 6 ? (threadIdx.x - 32) % 256 : threadIdx.x - 32;
            for (int i = t0; i < nv; i += gthreads) {
                const uint4 v = p[i];
                acc += v.x ^ v.w;
                if (mode >= 5) {
                    const float f = __uint_as_float((v.y & 0x007fffffu) | 0x3f800000u);
                    for (int k = 0; k < work; k++) facc = fmaf(facc, 0.999f, f);
                }
            }
        }
        // every thread of the barrier (or warp) agrees on a timed-out wait
        if (mode == 1 || mode == 3 || mode == 5)
            ok = !group_sync_or(1, 512, !ok);  // the 16 consumer warps
        else if (mode == 6)
            ok = !group_sync_or(2 + grp, 256, !ok);  // this group of 8
        else
            ok = __all_sync(0xffffffffu, ok);
        if (!ok) {
            atomicExch(err, 2);
            stop = 1;
            break;
        }
        if (mode == 1 || mode == 3 || mode == 5) {
            if (threadIdx.x == 32) arrive(&empty[st]);
        } else if (mode == 6) {
            if ((threadIdx.x - 32) % 256 == 0) arrive(&empty[st]);
        } else if (lane == 0) {
            arrive(&empty[st]);
        }
    }
    if (acc == 0x12345678u || facc == 1.2345f) atomicAdd(err, 4);  // keeps the reads
}

int main() {
    const size_t total = (size_t)4 << 30;
    uint8_t* src;
    int* err;
    if (cudaMalloc(&src, total) != cudaSuccess || cudaMalloc(&err, 4) != cudaSuccess) return 1;
    cudaMemset(src, 1, total);
    cudaMemset(err, 0, 4);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    cudaFuncSetAttribute(k_ring, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
    struct C {
        int S, slot, per_sm, ef, mode, work;
    } cs[] = {
        {4, 18432, 1, 1, 0, 0},  {8, 18432, 1, 1, 0, 0},  {11, 18432, 1, 1, 0, 0},
        {8, 18432, 1, 0, 0, 0},  {16, 9216, 1, 1, 0, 0},  {24, 4608, 1, 1, 0, 0},
        {4, 36864, 1, 1, 0, 0},  {4, 18432, 2, 1, 0, 0},  {8, 18432, 1, 1, 1, 0},
        {8, 18432, 1, 1, 2, 0},  {8, 18432, 1, 1, 3, 0},  {8, 18432, 1, 1, 4, 0},
        {4, 36864, 1, 1, 3, 0},  {16, 9216, 1, 1, 3, 0},  {8, 18432, 1, 1, 5, 16},
        {8, 18432, 1, 1, 6, 16}, {4, 36864, 1, 1, 5, 16}, {4, 36864, 1, 1, 6, 16},
    };
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    for (const C& c : cs) {
        const int grid = sms * c.per_sm;
        const size_t per_cta = (total / grid) / c.slot * c.slot;
        const size_t smem = (size_t)c.S * c.slot;
        const int threads = c.mode ? 544 : 64;
        float ms = 0.f;
        cudaError_t e = cudaSuccess;
        for (int rep = 0; rep < 2; rep++) {  // the second run is reported
            cudaEventRecord(e0);
            k_ring<<<grid, threads, smem>>>(src, per_cta, c.S, c.slot, err, c.ef, c.mode, c.work);
            cudaEventRecord(e1);
            e = cudaDeviceSynchronize();
            cudaEventElapsedTime(&ms, e0, e1);
        }
        int h_err = 0;
        cudaMemcpy(&h_err, err, 4, cudaMemcpyDeviceToHost);
        printf("mode %d work %2d: %2d x %6d B slots, %d CTA/SM (%3zu KB in flight per SM)%s: "
               "%7.1f GB/s  [%s, err %d]\n",
               c.mode, c.work, c.S, c.slot, c.per_sm, (size_t)c.S * c.slot * c.per_sm / 1024,
               c.ef ? "" : " evict_normal", (double)per_cta * grid / (ms * 1e-3) / 1e9,
               cudaGetErrorString(e), h_err);
    }
    return 0;
}
