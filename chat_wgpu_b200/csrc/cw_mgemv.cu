// cw_mgemv.cu -- the co-batched decode GEMV: Y[s] = W X[s] for the sessions
// s of a session group (up to 8), with the Q4_0 weights streamed from HBM
// ONCE for all of them.  Used by the group step (cw_prefill.cu) in place of
// the tensor-core GEMM + split-K reduce when the group is small: at 8 rows
// the GEMM pays ~18 us of pipeline fill and drain per projection, while this
// kernel is one pass over the weight stream.
//
// Data movement: as the streaming GEMV (cw_gemv.cuh): chunks of RC
// consecutive rows (payload + f16 scales, two cp.async.bulk copies) through a
// ring of S shared-memory stages, the first S issued before
// griddepcontrol.wait; one CTA per SM (16 warps).
//
// Work mapping: lane L of a warp serves session s = L % BT of the CTA's
// session set and block lane j = L / BT; WPR warps share a row, so a row's
// blocks b = (warp % WPR) * J + j + k * WPR * J (k < BPL, J = 32 / BT) are
// covered with every lane holding ITS session's q24 planes (cw_device.cuh)
// of its BPL blocks in registers.  The BT lanes of a block read the same
// shared-memory weight words (a broadcast), so the stream is read from
// shared memory once per warp.  A row's per-session partials are summed over
// the J block lanes by shuffles and over the WPR warps through shared memory
// in a fixed order, so results are bit-reproducible run to run.
//
// Prologue: PRO_NORM forms each session's rmsnorm (norm.wgsl:20-56) inside
// the kernel (sums of squares over 512/BT threads per session, fixed order);
// then the CTA converts every (session, block) of its inputs once into q24
// planes in shared memory, four elements per lane (q24_quad), and each lane
// loads the planes of its own blocks into registers.
//
// Waits are bounded by %globaltimer: a timed-out wait records DEV_TIMEOUT,
// waits (bounded) for the copies in flight and ends the kernel.
#include <algorithm>
#include <map>
#include <tuple>

#include "cw_gemv.cuh"
#include "cw_mgemv.h"

namespace cw {

constexpr int MG_THREADS = 512;
constexpr int MG_WARPS = MG_THREADS / 32;

template <int BT_, int WPR_, int BPL_, int RPW_>
struct MgCfg {
    static constexpr int BT = BT_, WPR = WPR_, BPL = BPL_, RPW = RPW_;
    static constexpr int J = 32 / BT;  // block lanes per warp (lanes of one session)
    static constexpr int SLOTS = MG_WARPS / WPR;
    static constexpr int RC = SLOTS * RPW;  // rows per chunk
    static constexpr int NB_MAX = WPR * J * BPL;
    static_assert(RC % 2 == 0, "gate/up pairs lie in one chunk");
};
// 5..8 sessions
using Mg8a = MgCfg<8, 4, 2, 4>;   // K <= 1024: 16 rows per chunk
using Mg8b = MgCfg<8, 8, 2, 4>;   // K <= 2048:  8 rows
using Mg8c = MgCfg<8, 16, 2, 4>;  // K <= 4096:  4 rows
// 1..4 sessions (and 5..8 sessions in two session sets for K > 4096)
using Mg4a = MgCfg<4, 2, 2, 4>;   // K <= 1024: 32 rows
using Mg4b = MgCfg<4, 4, 2, 4>;   // K <= 2048: 16 rows
using Mg4c = MgCfg<4, 8, 2, 4>;   // K <= 4096:  8 rows
using Mg4d = MgCfg<4, 16, 3, 2>;  // K <= 12288: 2 rows

__device__ __forceinline__ int ld_volatile_shared(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

__device__ __forceinline__ float mg_ss4(const float4& v, float ss) {
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    return fmaf(v.w, v.w, ss);
}

// sum_j (q_j - 8) X_j of one Q4_0 block against one q24 block (six
// independent dp4a chains, low and high nibbles apart).
__device__ __forceinline__ float mg_block_dot(const uint4& w4, const uint4 (&xa)[3],
                                              const uint4 (&xb)[3], int cb) {
    const unsigned w[4] = {w4.x, w4.y, w4.z, w4.w};
    const unsigned a0[4] = {xa[0].x, xa[0].y, xa[0].z, xa[0].w};
    const unsigned b0[4] = {xb[0].x, xb[0].y, xb[0].z, xb[0].w};
    const unsigned a1[4] = {xa[1].x, xa[1].y, xa[1].z, xa[1].w};
    const unsigned b1[4] = {xb[1].x, xb[1].y, xb[1].z, xb[1].w};
    const unsigned a2[4] = {xa[2].x, xa[2].y, xa[2].z, xa[2].w};
    const unsigned b2[4] = {xb[2].x, xb[2].y, xb[2].z, xb[2].w};
    int s0l = 0, s0h = 0, s1l = 0, s1h = 0, s2l = 0, s2h = 0;
#pragma unroll
    for (int t = 0; t < 4; t++) {
        const unsigned lo = w[t] & 0x0f0f0f0fu;
        const unsigned hi = (w[t] >> 4) & 0x0f0f0f0fu;
        s0l = dp4a_uu(lo, a0[t], s0l);
        s0h = dp4a_uu(hi, b0[t], s0h);
        s1l = dp4a_uu(lo, a1[t], s1l);
        s1h = dp4a_uu(hi, b1[t], s1h);
        s2l = dp4a_us(lo, a2[t], s2l);
        s2h = dp4a_us(hi, b2[t], s2h);
    }
    const int s01 = (s0l + s0h) + ((s1l + s1h) << 8) - cb;
    return fmaf((float)(s2l + s2h), 65536.0f, (float)s01);
}

__host__ __device__ constexpr size_t mg_pay_bytes(int RC, int nb) { return al128((size_t)RC * nb * 16); }
__host__ __device__ constexpr size_t mg_stage_bytes(int RC, int nb) {
    return mg_pay_bytes(RC, nb) + al128((size_t)RC * nb * 2);
}
template <class CF>
__host__ __device__ constexpr size_t mg_red_bytes() {
    return al16((size_t)2 * CF::RC * CF::WPR * CF::BT * 4);
}
// q24 planes of the BT sessions' inputs, one Q24 region per session
__host__ __device__ constexpr size_t mg_planes_bytes(int BT, int nb) {
    return (size_t)BT * al16(q24_bytes(nb));
}

template <class CF, int PRO, int EPI>
__global__ void __launch_bounds__(MG_THREADS, 1) k_mgemv(MgArgs a, int S) {
    constexpr int BT = CF::BT, WPR = CF::WPR, BPL = CF::BPL, RPW = CF::RPW, RC = CF::RC,
                  J = CF::J;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ float red[MG_WARPS];
    __shared__ float inv_s[BT];
    const int nb = a.K / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ls = lane % BT, lj = lane / BT;  // this lane's session (in the set) and block lane
    const int wsub = warp % WPR, slot = warp / WPR;
    const int s0 = blockIdx.y * BT;            // first session of this CTA's set
    const int ns = min(BT, a.B - s0);
    const long nchunks = ((long)a.N + RC - 1) / RC;
    const int mycount =
        blockIdx.x < nchunks ? (int)((nchunks - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    const size_t pay_b = mg_pay_bytes(RC, nb), stage_b = mg_stage_bytes(RC, nb);
    const size_t qreg = al16(q24_bytes(nb));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    unsigned char* planes = smem + 128;
    float* rbuf = reinterpret_cast<float*>(planes + (size_t)BT * qreg);
    unsigned char* stages = reinterpret_cast<unsigned char*>(rbuf) + mg_red_bytes<CF>();

    auto issue = [&](int i) {  // chunk i of this CTA into stage i % S (thread 0 only)
        const long c = blockIdx.x + (long)i * gridDim.x;
        const int st = i % S;
        const long row0 = c * RC;
        const int rows = (int)min((long)RC, (long)a.N - row0);
        const unsigned pb = (unsigned)rows * nb * 16, sb = (unsigned)rows * nb * 2;
        const uint64_t pol = l2_evict_first();
        fence_proxy_async();
        mbar_expect_tx(&bars[st], pb + sb);
        bulk_g2s_hint(stages + (size_t)st * stage_b, a.payload + (size_t)row0 * nb * 16, pb,
                      &bars[st], pol);
        bulk_g2s_hint(stages + (size_t)st * stage_b + pay_b, a.scales + (size_t)row0 * nb, sb,
                      &bars[st], pol);
    };
    if (tid == 0) {
        for (int st = 0; st < S; st++) mbar_init(&bars[st], 1);
        fence_mbar_init();
    }
    __syncthreads();
    // the weight stream does not depend on the previous kernel
    if (tid == 0)
        for (int i = 0; i < S && i < mycount; i++) issue(i);
    pdl_trigger();
    pdl_wait();

    // ---- prologue: per-session rmsnorm scale (PRO_NORM), then this lane's
    // blocks of its session's input as q24 planes in registers
    if constexpr (PRO == PRO_NORM) {
        constexpr int TPS = MG_THREADS / BT, WPS = TPS / 32;  // threads / warps per session
        const int ps = tid / TPS, pt = tid % TPS;
        float ss = 0.f;
        if (ps < ns) {
            const float* h = a.x + (size_t)(s0 + ps) * a.ldx;
#pragma unroll 4
            for (int i = 4 * pt; i < a.K; i += 4 * TPS)
                ss = mg_ss4(__ldcg(reinterpret_cast<const float4*>(h + i)), ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (tid < BT) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < WPS; w++) t += red[tid * WPS + w];
            inv_s[tid] = 1.0f / sqrtf(t / (float)a.K + a.eps);
        }
        __syncthreads();
    }
    // every (session, block) of the CTA's inputs converted once: four
    // consecutive elements per lane (q24_quad), one warp item = four blocks
    // of one session, coalesced 512-byte loads
    {
        const int nq = nb / 4, items = ns * nq;
        const int sub = lane >> 3, e0 = 4 * (lane & 7);
        for (int it = warp; it < items; it += MG_WARPS) {
            const int s = it / nq, b = 4 * (it - s * nq) + sub, i = b * 32 + e0;
            float4 v = __ldcg(reinterpret_cast<const float4*>(a.x + (size_t)(s0 + s) * a.ldx + i));
            if constexpr (PRO == PRO_NORM) {
                const float inv = inv_s[s];
                float4 g = __ldg(reinterpret_cast<const float4*>(a.norm_w + i));
                if (a.unit) g = make_float4(1.0f + g.x, 1.0f + g.y, 1.0f + g.z, 1.0f + g.w);
                v = make_float4(__fmul_rn(__fmul_rn(v.x, inv), g.x), __fmul_rn(__fmul_rn(v.y, inv), g.y),
                                __fmul_rn(__fmul_rn(v.z, inv), g.z), __fmul_rn(__fmul_rn(v.w, inv), g.w));
            }
            q24_quad(q24_carve(planes + (size_t)s * qreg, nb), b, true, v, lane);
        }
    }
    __syncthreads();
    // this lane's blocks of its session's planes, kept in registers
    uint4 xa[BPL][3], xb[BPL][3];
    int cb[BPL];
    float sbk[BPL];
    {
        const bool sv = ls < ns;
        const Q24 q = q24_carve(planes + (size_t)(sv ? ls : 0) * qreg, nb);
#pragma unroll
        for (int k = 0; k < BPL; k++) {
            const int b = wsub * J + lj + k * WPR * J;
            const bool in = sv && b < nb;
#pragma unroll
            for (int p = 0; p < 3; p++) {
                xa[k][p] = in ? q.pl[(p * 2 + 0) * nb + b] : make_uint4(0, 0, 0, 0);
                xb[k][p] = in ? q.pl[(p * 2 + 1) * nb + b] : make_uint4(0, 0, 0, 0);
            }
            cb[k] = in ? q.cb[b] : 0;
            sbk[k] = in ? q.sb[b] : 0.f;
        }
    }

    // ---- stream the chunks
    int failed = 0;
    for (int i = 0; i < mycount; i++) {
        const int st = i % S;
        const bool ok = mbar_wait(&bars[st], (unsigned)((i / S) & 1), GEMV_WAIT_NS);
        const unsigned char* pay = stages + (size_t)st * stage_b;
        const __half* scs = reinterpret_cast<const __half*>(pay + pay_b);
        const long row0 = (blockIdx.x + (long)i * gridDim.x) * RC;
        const int rows = (int)min((long)RC, (long)a.N - row0);
        float* rb = rbuf + (size_t)(i & 1) * RC * WPR * BT;
        float acc[RPW];
#pragma unroll
        for (int jr = 0; jr < RPW; jr++) acc[jr] = 0.f;
#pragma unroll
        for (int k = 0; k < BPL; k++) {
            const int b = wsub * J + lj + k * WPR * J;
            uint4 w4[RPW];
            float dd[RPW];
#pragma unroll
            for (int jr = 0; jr < RPW; jr++) {
                const int r = slot * RPW + jr;
                const bool in = b < nb && r < rows;
                const size_t blk = in ? (size_t)r * nb + b : 0;
                w4[jr] = in ? reinterpret_cast<const uint4*>(pay)[blk] : make_uint4(0, 0, 0, 0);
                dd[jr] = in ? __half2float(scs[blk]) : 0.f;
            }
#pragma unroll
            for (int jr = 0; jr < RPW; jr++)
                acc[jr] = fmaf(dd[jr] * sbk[k], mg_block_dot(w4[jr], xa[k], xb[k], cb[k]), acc[jr]);
        }
        // sum over the J block lanes of each session (lanes ls, ls + BT, ...)
#pragma unroll
        for (int jr = 0; jr < RPW; jr++) {
#pragma unroll
            for (int o = BT; o < 32; o <<= 1) acc[jr] += __shfl_xor_sync(FULL, acc[jr], o);
        }
        if (lj == 0) {
#pragma unroll
            for (int jr = 0; jr < RPW; jr++) rb[((slot * RPW + jr) * WPR + wsub) * BT + ls] = acc[jr];
        }
        if (__syncthreads_or(!ok)) {  // stage consumed, row partials complete
            failed = i + 1;
            break;
        }
        if (tid == 0 && i + S < mycount) issue(i + S);
        // epilogue: fixed-order sum of the WPR partials of each (row, session)
        if constexpr (EPI == EPI_GLU) {
            if (tid < (RC / 2) * BT) {
                const int pr = tid / BT, s = tid % BT, r0 = 2 * pr;
                if (s < ns && r0 + 1 < rows) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int w = 0; w < WPR; w++) {
                        gv += rb[(r0 * WPR + w) * BT + s];
                        uv += rb[((r0 + 1) * WPR + w) * BT + s];
                    }
                    const float act = a.geglu ? gelu_ref_f(gv) : silu_ref_f(gv);
                    a.y[(size_t)(s0 + s) * a.ldy + (row0 + r0) / 2] = act * uv;
                }
            }
        } else {
            if (tid < RC * BT) {
                const int r = tid / BT, s = tid % BT;
                if (s < ns && r < rows) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < WPR; w++) v += rb[(r * WPR + w) * BT + s];
                    const long row = row0 + r;
                    float* yp = a.y + (size_t)(s0 + s) * a.ldy + row;
                    if (EPI == EPI_RESID)
                        *yp = *yp + v;
                    else
                        *yp = a.bias ? v + a.bias[row] : v;
                }
            }
        }
    }
    if (failed && tid == 0) {
        // record the timeout and let every issued copy land before exiting
        atomicExch(a.status, (int)DEV_TIMEOUT);
        const int issued = min(mycount, failed - 1 + S);
        for (int i = failed - 1; i < issued; i++)
            mbar_wait(&bars[i % S], (unsigned)((i / S) & 1), GEMV_WAIT_NS);
    }
}

// ---- integer tensor-core variant (K <= 4096) ---------------------------------------
// The same products on the warp-level integer MMA (mma.sync m16n8k32, u8 x u8 /
// u8 x s8 -> s32): one MMA multiplies 16 weight rows' 4-bit codes (as bytes)
// of one Q4_0 block by one q24 byte plane of the 8 session columns, so a
// block costs three MMAs for 16 rows x 8 sessions instead of 24 dp4a per
// (row, session).  The integer sums equal the dp4a ones exactly, and they
// are combined per (row, session, block) as there: T = D0 + 256 D1 - 8 sum X
// + 65536 D2, acc += d * 2^(e-22) * T.
//
// Weights: a tile-interleaved copy of the matrix (mg_tile_pack): per 16-row
// tile its payload [block][row][16 B] then its scales [block][row], one
// contiguous range, so a tile is ONE bulk copy and a warp's A-fragment loads
// (word c of a block in rows g and g + 8) and scale loads hit distinct
// banks.  The session inputs are converted once per CTA into q24 planes
// stored fragment-major (per block, session and thread-in-group the six
// B-fragment words, then (8 sum X, 2^(e-22)) pairs), so a block's B operands
// are three conflict-free 8-byte loads and one 16-byte load.
//
// Work: the 16 compute warps form 16 / WG groups of WG warps; a group takes
// a tile, each of its warps a 1/WG share of the blocks, and the group's
// partial sums meet in shared memory behind a named barrier of the group
// (which also agrees on a timed-out wait).  Tile q of the CTA goes to group
// q % NG and ring stage q % S (S a multiple of NG, so every stage belongs to
// one group).  A 17th warp only streams the tiles, refilling a stage once
// its group released it (the stage's "empty" mbarrier).
constexpr int MI_RC = 16;                      // rows per tile
constexpr int MI_BLOCK = MG_THREADS + 32;      // + the producer warp
constexpr int MI_SMAX = 16;                    // ring stages at most
constexpr int MI_IB = 4;                       // prologue items per warp and load batch

__device__ __forceinline__ void mma_u8u8(int (&d)[4], const unsigned (&a)[4], unsigned b0,
                                         unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}
__device__ __forceinline__ void mma_u8s8(int (&d)[4], const unsigned (&a)[4], unsigned b0,
                                         unsigned b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0));
}
// named barrier 1 over the 16 compute warps
__device__ __forceinline__ void mi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(MG_THREADS) : "memory"); }
// named barrier `id` over `n` threads; returns whether any passed v != 0
__device__ __forceinline__ bool mi_group_sync_or(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

// one tile of the tile-interleaved copy: 16 rows x nb blocks x 18 bytes
__host__ __device__ constexpr size_t mi_tile_bytes(int nb) { return (size_t)MI_RC * nb * 18; }
// fragment-major planes: words [nb][8 sessions][4 c][6], then int2 [nb][8]
__host__ __device__ constexpr size_t mi_frag_bytes(int nb) { return (size_t)nb * (768 + 64); }
// row partials [group][2][warp in group][MT * 16 rows][session]
__host__ __device__ constexpr size_t mi_red_bytes(int MT) { return (size_t)2 * MG_WARPS * MI_RC * MT * 8 * 4; }

struct MiShared {
    uint64_t full[MI_SMAX], empty[MI_SMAX];
    int abort, issued, prod_done;
};

// Tile t of a Q4_0 matrix (payload [N][nb][16], scales [N][nb]) into the
// tile-interleaved layout; rows past N are zeros (scale 0).
__global__ void k_mg_pack(const uint8_t* __restrict__ payload, const __half* __restrict__ scales,
                          int N, int nb, uint8_t* __restrict__ dst) {
    const long t = blockIdx.x;
    uint8_t* tp = dst + (size_t)t * mi_tile_bytes(nb);
    uint4* pay = reinterpret_cast<uint4*>(tp);
    __half* sc = reinterpret_cast<__half*>(tp + (size_t)MI_RC * nb * 16);
    for (int i = threadIdx.x; i < MI_RC * nb; i += blockDim.x) {
        const int b = i / MI_RC, r = i % MI_RC;
        const long row = t * MI_RC + r;
        const bool in = row < N;
        pay[i] = in ? reinterpret_cast<const uint4*>(payload)[(size_t)row * nb + b] : make_uint4(0, 0, 0, 0);
        sc[i] = in ? scales[(size_t)row * nb + b] : __float2half(0.0f);
    }
}

template <int WG, int MT, int PRO, int EPI>
__global__ void __launch_bounds__(MI_BLOCK, 1) k_mgemm(MgArgs a, int S) {
    constexpr int NG = MG_WARPS / WG;  // warp groups (stages being consumed per CTA)
    constexpr int RS = MI_RC * MT;     // rows per stage: MT MMA tiles
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ MiShared sh;
    __shared__ float red[MG_WARPS];
    __shared__ float inv_s[8];
    const int nb = a.K / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int ns = min(8, a.B);
    const long ntiles = ((long)a.N + MI_RC - 1) / MI_RC;
    const long nstage = (ntiles + MT - 1) / MT;  // stage loads of MT tiles
    const int mycount = blockIdx.x < nstage ? (int)((nstage - 1 - blockIdx.x) / gridDim.x + 1) : 0;
    const size_t tile_b = mi_tile_bytes(nb), stage_b = al128(MT * tile_b);
    uint32_t* frag = reinterpret_cast<uint32_t*>(smem);
    int2* cbsb = reinterpret_cast<int2*>(smem + (size_t)nb * 768);
    float* rbuf = reinterpret_cast<float*>(smem + al128(mi_frag_bytes(nb)));
    unsigned char* stages = reinterpret_cast<unsigned char*>(rbuf) + mi_red_bytes(MT);

    if (tid == 0) {
        for (int st = 0; st < S; st++) {
            mbar_init(&sh.full[st], 1);
            mbar_init(&sh.empty[st], 1);
        }
        fence_mbar_init();
        sh.abort = 0;
        sh.issued = 0;
        sh.prod_done = 0;
    }
    __syncthreads();
    if (warp == MG_WARPS) {
        // ---- the producer: stage load q (MT tiles) into stage q % S once that stage's
        // previous tile (q - S) was released.  The weight stream does not
        // depend on the previous kernel.
        pdl_trigger();
        if (lane == 0) {
            const uint64_t pol = l2_evict_first();
            int q = 0;
            for (; q < mycount; q++) {
                const int st = q % S;
                if (q >= S) {
                    const unsigned par = (unsigned)(((q / S) - 1) & 1);
                    bool ok = mbar_try_wait(&sh.empty[st], par);
                    const uint64_t t0 = ok ? 0 : global_ns();
                    while (!ok) {
                        if (ld_volatile_shared(&sh.abort) || global_ns() - t0 > GEMV_WAIT_NS) break;
                        ok = mbar_try_wait(&sh.empty[st], par);
                    }
                    if (!ok) break;
                }
                const long t0 = (blockIdx.x + (long)q * gridDim.x) * MT;  // first tile
                const unsigned bytes = (unsigned)(min((long)MT, ntiles - t0) * tile_b);
                mbar_expect_tx(&sh.full[st], bytes);
                bulk_g2s_hint(stages + (size_t)st * stage_b, a.tiles + (size_t)t0 * tile_b, bytes,
                              &sh.full[st], pol);
            }
            sh.issued = q;
            __threadfence_block();
            *reinterpret_cast<volatile int*>(&sh.prod_done) = 1;
        }
        return;
    }
    pdl_wait();

    // ---- prologue: per-session rmsnorm scales, then every (session, block)
    // of the inputs as q24 planes, fragment-major; sessions >= ns are zeros
    if constexpr (PRO == PRO_NORM) {
        constexpr int TPS = MG_THREADS / 8, WPS = TPS / 32;  // 64 threads per session
        const int ps = tid / TPS, pt = tid % TPS;
        float ss = 0.f;
        if (ps < ns) {
            const float* h = a.x + (size_t)ps * a.ldx;
#pragma unroll 4
            for (int i = 4 * pt; i < a.K; i += 4 * TPS)
                ss = mg_ss4(__ldcg(reinterpret_cast<const float4*>(h + i)), ss);
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        mi_sync();
        if (tid < 8) {
            float t = 0.f;
#pragma unroll
            for (int w = 0; w < WPS; w++) t += red[tid * WPS + w];
            inv_s[tid] = 1.0f / sqrtf(t / (float)a.K + a.eps);
        }
        mi_sync();
    }
    {
        // item = (session s, four blocks 4t..4t+3); lane: block 4t + lane/8,
        // half h = (lane/4) & 1, word c = lane & 3 -> elements 16h + 4c .. +3.
        // Items in batches of MI_IB per warp, every load of a batch issued
        // before any is used (one L2 round trip per batch, not per item).
        const int nq = nb / 4, items = 8 * nq;
        const int sub = lane >> 3, hh = (lane >> 2) & 1, cc = lane & 3;
        for (int it0 = warp; it0 < items; it0 += MI_IB * MG_WARPS) {
            float4 vv[MI_IB], ww[MI_IB];
#pragma unroll
            for (int u = 0; u < MI_IB; u++) {
                const int it = it0 + u * MG_WARPS;
                const int s = it / nq, b = 4 * (it - s * nq) + sub, i = b * 32 + 16 * hh + 4 * cc;
                const bool in = it < items && s < ns;  // warp-uniform
                vv[u] = in ? __ldcg(reinterpret_cast<const float4*>(a.x + (size_t)s * a.ldx + i))
                           : make_float4(0.f, 0.f, 0.f, 0.f);
                if constexpr (PRO == PRO_NORM)
                    ww[u] = in ? __ldg(reinterpret_cast<const float4*>(a.norm_w + i))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < MI_IB; u++) {
                const int it = it0 + u * MG_WARPS;
                if (it >= items) break;  // warp-uniform
                const int s = it / nq, b = 4 * (it - s * nq) + sub;
                float4 v = vv[u];
                if constexpr (PRO == PRO_NORM) {
                    const float inv = inv_s[s];
                    float4 w = ww[u];
                    if (a.unit) w = make_float4(1.0f + w.x, 1.0f + w.y, 1.0f + w.z, 1.0f + w.w);
                    v = make_float4(__fmul_rn(__fmul_rn(v.x, inv), w.x), __fmul_rn(__fmul_rn(v.y, inv), w.y),
                                    __fmul_rn(__fmul_rn(v.z, inv), w.z), __fmul_rn(__fmul_rn(v.w, inv), w.w));
                }
                // block max and integer sum over the block's 8 lanes (q24_quad's scheme)
                unsigned m = max(max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))),
                                 max(__float_as_uint(fabsf(v.z)), __float_as_uint(fabsf(v.w))));
                m = max(m, __shfl_xor_sync(FULL, m, 1));
                m = max(m, __shfl_xor_sync(FULL, m, 2));
                m = max(m, __shfl_xor_sync(FULL, m, 4));
                int X0, X1, X2, X3;
                float sb;
                q24_scale(m, v.x, X0, sb);
                q24_scale(m, v.y, X1, sb);
                q24_scale(m, v.z, X2, sb);
                q24_scale(m, v.w, X3, sb);
                uint32_t* fw = frag + ((size_t)(b * 8 + s) * 4 + cc) * 6 + hh;
#pragma unroll
                for (int pl = 0; pl < 3; pl++) {
                    const unsigned sel = (unsigned)pl | ((4u + pl) << 4);
                    const unsigned lo = __byte_perm((unsigned)X0, (unsigned)X1, sel);
                    const unsigned hi = __byte_perm((unsigned)X2, (unsigned)X3, sel);
                    fw[2 * pl] = __byte_perm(lo, hi, 0x5410);
                }
                int sx = (X0 + X1) + (X2 + X3);
                sx += __shfl_xor_sync(FULL, sx, 1);
                sx += __shfl_xor_sync(FULL, sx, 2);
                sx += __shfl_xor_sync(FULL, sx, 4);
                if ((lane & 7) == 0) cbsb[b * 8 + s] = make_int2(8 * sx, __float_as_int(sb));
            }
        }
    }
    mi_sync();

    // ---- this group's stage loads: j, j + NG, ... of the CTA's
    const int j = warp / WG, wg = warp % WG, gt = tid - j * WG * 32;  // group, warp and thread in it
    const int spg = S / NG;                                            // ring stages per group
    const int g = lane >> 2, c = lane & 3;  // MMA group (row / session column), thread in group
    float* rgrp = rbuf + (size_t)j * 2 * WG * RS * 8;
    int k = 0;  // tiles consumed by the group
    bool bad = false;
    unsigned long long best = argmax_key_init();  // EPI_HEAD: this thread's session's best key
    for (int q = j; q < mycount; q += NG, k++) {
        const int st = j + (k % spg) * NG;
        const bool ok = mbar_wait(&sh.full[st], (unsigned)((k / spg) & 1), GEMV_WAIT_NS);
        const unsigned char* pay = stages + (size_t)st * stage_b;
        const long row0 = (blockIdx.x + (long)q * gridDim.x) * RS;
        const int rows = (int)min((long)RS, (long)a.N - row0);
        float acc[MT][4];
#pragma unroll
        for (int t = 0; t < MT; t++)
#pragma unroll
            for (int e = 0; e < 4; e++) acc[t][e] = 0.f;
#pragma unroll 2
        for (int b = wg; b < nb; b += WG) {
            // the block's B operands, shared by the MT tiles of the stage
            const uint32_t* fb = frag + ((size_t)(b * 8 + g) * 4 + c) * 6;
            const uint2 x0 = *reinterpret_cast<const uint2*>(fb);
            const uint2 x1 = *reinterpret_cast<const uint2*>(fb + 2);
            const uint2 x2 = *reinterpret_cast<const uint2*>(fb + 4);
            const int4 cs = *reinterpret_cast<const int4*>(cbsb + b * 8 + 2 * c);
            const int cb[2] = {cs.x, cs.z};
            const float sbv[2] = {__int_as_float(cs.y), __int_as_float(cs.w)};
#pragma unroll
            for (int t = 0; t < MT; t++) {
                const unsigned char* tp = pay + (size_t)t * tile_b;  // rows past N: zero tiles
                const unsigned char* scs = tp + (size_t)MI_RC * nb * 16;
                const unsigned w0 = *reinterpret_cast<const unsigned*>(tp + ((size_t)b * MI_RC + g) * 16 + 4 * c);
                const unsigned w1 = *reinterpret_cast<const unsigned*>(tp + ((size_t)b * MI_RC + g + 8) * 16 + 4 * c);
                const float d0 = __half2float(*reinterpret_cast<const __half*>(scs + ((size_t)b * MI_RC + g) * 2));
                const float d1 = __half2float(*reinterpret_cast<const __half*>(scs + ((size_t)b * MI_RC + g + 8) * 2));
                const unsigned af[4] = {w0 & 0x0f0f0f0fu, w1 & 0x0f0f0f0fu, (w0 >> 4) & 0x0f0f0f0fu,
                                        (w1 >> 4) & 0x0f0f0f0fu};
                int D0[4], D1[4], D2[4];
                mma_u8u8(D0, af, x0.x, x0.y);
                mma_u8u8(D1, af, x1.x, x1.y);
                mma_u8s8(D2, af, x2.x, x2.y);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int h = e & 1;
                    const int s01 = D0[e] + (D1[e] << 8) - cb[h];
                    const float T = fmaf((float)D2[e], 65536.0f, (float)s01);
                    acc[t][e] = fmaf((e < 2 ? d0 : d1) * sbv[h], T, acc[t][e]);
                }
            }
        }
        // this warp's partial sums: rows 16t + g, 16t + g + 8 x sessions 2c, 2c + 1
        float* rb = rgrp + (size_t)(k & 1) * WG * RS * 8;
        float* rw = rb + (size_t)wg * RS * 8;
#pragma unroll
        for (int t = 0; t < MT; t++) {
            *reinterpret_cast<float2*>(rw + (16 * t + g) * 8 + 2 * c) = make_float2(acc[t][0], acc[t][1]);
            *reinterpret_cast<float2*>(rw + (16 * t + g + 8) * 8 + 2 * c) = make_float2(acc[t][2], acc[t][3]);
        }
        if (mi_group_sync_or(2 + j, WG * 32, !ok)) {  // stage read, partial sums complete
            bad = true;
            break;
        }
        if (gt == 0)  // hand the stage back to the producer
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&sh.empty[st]))
                         : "memory");
        // epilogue: fixed-order sum of the group's WG partials of each (row, session)
        if constexpr (EPI == EPI_GLU) {
            if (gt < (RS / 2) * 8) {
                const int pr = gt >> 3, s = gt & 7, r0 = 2 * pr;
                if (s < ns && r0 + 1 < rows) {
                    float gv = 0.f, uv = 0.f;
#pragma unroll
                    for (int w = 0; w < WG; w++) {
                        gv += rb[((size_t)w * RS + r0) * 8 + s];
                        uv += rb[((size_t)w * RS + r0 + 1) * 8 + s];
                    }
                    const float act = a.geglu ? gelu_ref_f(gv) : silu_ref_f(gv);
                    a.y[(size_t)s * a.ldy + (row0 + r0) / 2] = act * uv;
                }
            }
        } else {
            for (int o = gt; o < RS * 8; o += WG * 32) {
                const int r = o >> 3, s = o & 7;
                if (s < ns && r < rows) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < WG; w++) v += rb[((size_t)w * RS + r) * 8 + s];
                    const long row = row0 + r;
                    if constexpr (EPI == EPI_HEAD) {
                        if (a.softcap > 0.f) v = a.softcap * tanhf(v / a.softcap);
                        a.yrow[s][row] = v;
                        const unsigned long long kk = argmax_key(v, (unsigned)row);
                        best = kk > best ? kk : best;
                    } else {
                        float* yp = a.y + (size_t)s * a.ldy + row;
                        if (EPI == EPI_RESID)
                            *yp = *yp + v;
                        else
                            *yp = a.bias ? v + a.bias[row] : v;
                    }
                }
            }
        }
    }
    if constexpr (EPI == EPI_HEAD) {
        // per session: the CTA's best argmax key (the threads of session s
        // are those with tid % 8 == s), one atomicMax per session and CTA
        __shared__ unsigned long long kbuf[MG_WARPS][8];
        unsigned long long t8 = __shfl_xor_sync(FULL, best, 8);
        best = t8 > best ? t8 : best;
        t8 = __shfl_xor_sync(FULL, best, 16);
        best = t8 > best ? t8 : best;
        if (lane < 8) kbuf[warp][lane] = best;
        mi_sync();
        if (tid < ns && !bad) {
            unsigned long long kk = kbuf[0][tid];
            for (int w = 1; w < MG_WARPS; w++) kk = kbuf[w][tid] > kk ? kbuf[w][tid] : kk;
            atomicMax(a.keys + tid, kk);
        }
    }
    if (bad && gt == 0) {
        // record the timeout, stop the producer, and let every tile it issued
        // into this group's stages land before the group exits (bounded waits)
        atomicExch(a.status, (int)DEV_TIMEOUT);
        *reinterpret_cast<volatile int*>(&sh.abort) = 1;
        const uint64_t t0 = global_ns();
        while (!ld_volatile_shared(&sh.prod_done) && global_ns() - t0 < GEMV_WAIT_NS) {
        }
        const int issued = ld_volatile_shared(&sh.issued);
        const int mine = issued > j ? (issued - j + NG - 1) / NG : 0;
        for (int kk = k; kk < mine; kk++)
            mbar_wait(&sh.full[j + (kk % spg) * NG], (unsigned)((kk / spg) & 1), GEMV_WAIT_NS);
    }
}

// ---- host side --------------------------------------------------------------------
template <class CF, int PRO, int EPI>
static int mg_go(cw_ctx* ctx, const MgArgs& a, int sets, bool pdl) {
    const int nb = a.K / 32;
    const long nchunks = ((long)a.N + CF::RC - 1) / CF::RC;
    auto kern = k_mgemv<CF, PRO, EPI>;
    const size_t stage_b = mg_stage_bytes(CF::RC, nb);
    // (1 KB kept for the kernel's static shared memory)
    const size_t fixed = 128 + mg_planes_bytes(CF::BT, nb) + mg_red_bytes<CF>() + 1024;
    // one CTA per SM per session set; as many ring stages as this CTA has
    // chunks (all of a small GEMV's weights in flight at once), up to the
    // shared memory the SM offers
    const long grid_x = std::max<long>(1, std::min<long>(nchunks, ctx->sm_count / sets));
    const long per_cta = (nchunks + grid_x - 1) / grid_x;
    const int s_fit = (int)std::min<size_t>(16, ((size_t)ctx->max_smem_optin - fixed) / stage_b);
    CW_CHECK(s_fit >= 1, CW_ERR_UNSUPPORTED, "mgemv: K=%d chunk does not fit shared memory", a.K);
    const int S = (int)std::max<long>(1, std::min<long>(per_cta, s_fit));
    const size_t smem = fixed - 1024 + (size_t)S * stage_b;
    static thread_local std::map<std::pair<int, const void*>, size_t> attr_set;
    const auto key = std::make_pair(ctx->device, (const void*)kern);
    auto it = attr_set.find(key);
    if (it == attr_set.end() || it->second < smem) {
        CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set[key] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid_x, (unsigned)sets);
    cfg.blockDim = dim3(MG_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    MgArgs args = a;
    if (!args.status) args.status = ctx->d_status;
    CW_CUDA(cudaLaunchKernelEx(&cfg, kern, args, S));
    return CW_OK;
}

template <int WG, int MT, int PRO, int EPI>
static int mi_go(cw_ctx* ctx, const MgArgs& a, bool pdl) {
    constexpr int NG = MG_WARPS / WG;
    const int nb = a.K / 32;
    CW_CHECK(a.tiles, CW_ERR_INVALID_ARG, "mgemm: no tile-interleaved weight copy");
    const long ntiles = ((long)a.N + MI_RC - 1) / MI_RC;
    const long nstage = (ntiles + MT - 1) / MT;
    auto kern = k_mgemm<WG, MT, PRO, EPI>;
    const size_t stage_b = al128(MT * mi_tile_bytes(nb));
    // (1 KB kept for the kernel's static shared memory)
    const size_t fixed = al128(mi_frag_bytes(nb)) + mi_red_bytes(MT) + 1024;
    const long grid_x = std::max<long>(1, std::min<long>(nstage, ctx->sm_count));
    const long per_cta = (nstage + grid_x - 1) / grid_x;
    // ring stages: a multiple of the group count, enough for this CTA's tiles
    const int s_fit = (int)std::min<size_t>(MI_SMAX, ((size_t)ctx->max_smem_optin - fixed) / stage_b);
    CW_CHECK(s_fit >= NG, CW_ERR_UNSUPPORTED, "mgemm: K=%d tiles do not fit shared memory", a.K);
    const int S = (int)std::min<long>(s_fit / NG, (per_cta + NG - 1) / NG) * NG;
    const size_t smem = fixed - 1024 + (size_t)S * stage_b;
    static thread_local std::map<std::pair<int, const void*>, size_t> attr_set;
    const auto key = std::make_pair(ctx->device, (const void*)kern);
    auto it = attr_set.find(key);
    if (it == attr_set.end() || it->second < smem) {
        CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        attr_set[key] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid_x);
    cfg.blockDim = dim3(MI_BLOCK);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    MgArgs args = a;
    if (!args.status) args.status = ctx->d_status;
    CW_CUDA(cudaLaunchKernelEx(&cfg, kern, args, S));
    return CW_OK;
}

template <int PRO, int EPI>
static int mg_cfg(cw_ctx* ctx, const MgArgs& a, bool pdl) {
    const int nb = a.K / 32;
    if (a.mma && nb <= 128) {
        // integer tensor cores.  Stage loads of at least ~18 KB (two tiles at
        // K <= 1024): every stage costs a wait and a group barrier, which
        // small copies do not amortise.  Warp groups sized by the stage loads
        // a CTA gets: all 16 warps on one load (the per-layer projections,
        // one or two loads per CTA), 8 on each of two, 4 on each of four
        // (the LM head's long stream)
        const int mt = nb <= 32 ? 2 : 1;
        const long nstage = ((long)a.N + MI_RC * mt - 1) / (MI_RC * mt);
        const long per_cta = (nstage + ctx->sm_count - 1) / ctx->sm_count;
        int wg = per_cta >= 4 ? 4 : per_cta >= 2 ? 8 : 16;
        // at least one ring stage per group must fit beside the planes
        const size_t stage_b = al128(mt * mi_tile_bytes(nb));
        const size_t fixed = al128(mi_frag_bytes(nb)) + mi_red_bytes(mt) + 1024;
        const long s_fit = ((long)ctx->max_smem_optin - (long)fixed) / (long)stage_b;
        while (wg < 16 && MG_WARPS / wg > s_fit) wg *= 2;
        if (mt == 2) {
            if (wg == 4) return mi_go<4, 2, PRO, EPI>(ctx, a, pdl);
            if (wg == 8) return mi_go<8, 2, PRO, EPI>(ctx, a, pdl);
            return mi_go<16, 2, PRO, EPI>(ctx, a, pdl);
        }
        if (wg == 4) return mi_go<4, 1, PRO, EPI>(ctx, a, pdl);
        if (wg == 8) return mi_go<8, 1, PRO, EPI>(ctx, a, pdl);
        return mi_go<16, 1, PRO, EPI>(ctx, a, pdl);
    }
    if constexpr (EPI == EPI_HEAD) {
        return set_error(CW_ERR_UNSUPPORTED, "mgemv: the head epilogue needs the integer-MMA path");
    } else {
        if (a.B > 4 && nb <= Mg8c::NB_MAX) {
            if (nb <= Mg8a::NB_MAX) return mg_go<Mg8a, PRO, EPI>(ctx, a, 1, pdl);
            if (nb <= Mg8b::NB_MAX) return mg_go<Mg8b, PRO, EPI>(ctx, a, 1, pdl);
            return mg_go<Mg8c, PRO, EPI>(ctx, a, 1, pdl);
        }
        const int sets = (a.B + 3) / 4;
        if (nb <= Mg4a::NB_MAX) return mg_go<Mg4a, PRO, EPI>(ctx, a, sets, pdl);
        if (nb <= Mg4b::NB_MAX) return mg_go<Mg4b, PRO, EPI>(ctx, a, sets, pdl);
        if (nb <= Mg4c::NB_MAX) return mg_go<Mg4c, PRO, EPI>(ctx, a, sets, pdl);
        return mg_go<Mg4d, PRO, EPI>(ctx, a, sets, pdl);
    }
}

bool mgemv_supported(int K, int B) {
    const int nb = K / 32;
    return B >= 1 && B <= 8 && K % 256 == 0 && nb <= Mg4d::NB_MAX;
}

int launch_mgemv(cw_ctx* ctx, int pro, int epi, const MgArgs& a, bool pdl) {
    CW_CHECK(mgemv_supported(a.K, a.B), CW_ERR_UNSUPPORTED,
             "mgemv: K=%d with %d sessions not handled", a.K, a.B);
    if (pro == PRO_NORM && epi == EPI_STORE) return mg_cfg<PRO_NORM, EPI_STORE>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_GLU) return mg_cfg<PRO_NORM, EPI_GLU>(ctx, a, pdl);
    if (pro == PRO_X && epi == EPI_RESID) return mg_cfg<PRO_X, EPI_RESID>(ctx, a, pdl);
    if (pro == PRO_X && epi == EPI_STORE) return mg_cfg<PRO_X, EPI_STORE>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_HEAD) return mg_cfg<PRO_NORM, EPI_HEAD>(ctx, a, pdl);
    return set_error(CW_ERR_UNSUPPORTED, "mgemv: prologue %d / epilogue %d not instantiated", pro,
                     epi);
}

}  // namespace cw

namespace cw {

size_t mg_tile_bytes(int rows, int K) {
    return (size_t)((rows + MI_RC - 1) / MI_RC) * mi_tile_bytes(K / 32);
}
// (a stage load of MT tiles copies only the tiles that exist)

int mg_tile_pack(cw_ctx* ctx, const uint8_t* payload, const __half* scales, int rows, int K,
                 void* dst) {
    CW_CHECK(K % 256 == 0 && rows > 0, CW_ERR_INVALID_ARG, "mg_tile_pack: K=%d rows=%d", K, rows);
    const int nt = (rows + MI_RC - 1) / MI_RC;
    k_mg_pack<<<nt, 256, 0, ctx->stream>>>(payload, scales, rows, K / 32, (uint8_t*)dst);
    return check_launch("mg_tile_pack");
}

}  // namespace cw
