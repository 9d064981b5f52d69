// cw_step.cuh -- device side of the persistent decode step (cw_step.cu).
//
// The step of src/model/qwen3.rs:128-191 + mod.rs:93-122 (embed, per layer
// norm+QKV, QK-norm+RoPE+attention, o-proj+residual, norm+gate/up+SwiGLU,
// down+residual, then norm+LM head+argmax and the next-input bookkeeping) runs
// as a list of stages inside ONE kernel with one CTA per SM (16 warps).
// Consecutive stages are separated by a grid-wide barrier (a monotonic 64-bit
// counter, bounded wait); no kernel boundary, launch latency or grid drain
// sits between stages.
//
// Weight streaming is decoupled from that dependency chain: every CTA knows
// which weight chunks (16 KB of consecutive rows) it will consume in all the
// GEMV stages of the step, in order.  Its thread 0 keeps an 8-slot ring of
// shared memory filled with cp.async.bulk copies of the NEXT chunks in that
// sequence, refilling a slot as soon as it is consumed, so copies for the
// following stages (about two layers ahead) are in flight while the CTA waits
// at a barrier.  The GEMV arithmetic is the q24 dp4a scheme of cw_gemv.cuh.
//
// Cross-CTA data (hidden, q/k/v, attention output, activations, partials) is
// read with ld.global.cg so a stale L1 line can never be used.  All waits are
// bounded by %globaltimer; a timeout sets the status word, every CTA drains
// its copies and leaves, and the host reports CW_ERR_TIMEOUT.
#pragma once

#include "cw_attn.cuh"
#include "cw_gemv.cuh"
#include "cw_model.h"
#include "cw_ops.h"

namespace cw {

// 16 compute warps and one producer warp that only queues the weight copies
// (MK_BLOCK threads per CTA).  The compute warps synchronise among themselves
// with named barrier 1 (mk_sync): the producer never waits on them except
// through the ring's "empty" mbarriers, so the copy issue -- a few hundred
// cycles per bulk copy -- never sits on the compute warps' critical path.
constexpr int MK_THREADS = 512;  // compute threads
constexpr int MK_WARPS = MK_THREADS / 32;
constexpr int MK_BLOCK = MK_THREADS + 32;
__device__ __forceinline__ void mk_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(MK_THREADS) : "memory");
}
// mk_sync that also returns whether any compute thread passed v != 0
__device__ __forceinline__ bool mk_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(MK_THREADS)
        : "memory");
    return r != 0;
}
constexpr int MK_SLOTS = 8;
constexpr int MK_SLOT_PAY = 16384;  // nibble payload of one chunk
constexpr int MK_SLOT_SC = 2048;    // its f16 scales
constexpr int MK_SLOT_BYTES = MK_SLOT_PAY + MK_SLOT_SC;
constexpr uint64_t MK_WAIT_NS = 2000000000ull;  // 2 s
// profile stamps per stage and CTA: [0..3] %globaltimer (stage start, end of
// prologue, end of main loop, end of work), [4..11] clock64 at the MK_CLK
// points of the GEMV stages
constexpr int MK_STAMPS = 16;
enum {
    CLK_START = 0,    // stage start (after the barrier)
    CLK_AHEAD = 1,    // descriptor two stages ahead requested, K/V prefetch issued
    CLK_LOADED = 2,   // prologue: global inputs arrived (NORM) / converted (X)
    CLK_NORMED = 3,   // prologue: CTA-wide sum of squares done
    CLK_Q24 = 4,      // prologue: q24 planes written
    CLK_REGS = 5,     // planes in registers (after the CTA barrier)
    CLK_MAIN = 6,     // chunk loop done
    CLK_END = 7,      // stage end
    CLK_N = 8,
    // first chunk of the main loop (extra points, reported separately)
    CLK_WAITED = 8,   // its weights are in shared memory
    CLK_SUMMED = 9,   // row partials complete (after the CTA barrier)
    CLK_ISSUED = 10,  // next copy issued
};

// GEMV work mapping for 16 warps (see cw_gemv.cuh): WPR warps per row, BPL
// blocks per lane, RPW rows per warp; RC rows per chunk spread over NS ring
// slots of RS = RC / NS rows each (RS * K/2 <= 16 KB).  Two-slot chunks halve
// the per-chunk wait / reduce / barrier overhead of stages where a CTA has
// several chunks (the LM head, the FFN's 64 gate/up rows).
template <int WPR_, int BPL_, int RPW_, int NS_ = 1>
struct MCfg {
    static constexpr int WPR = WPR_, BPL = BPL_, RPW = RPW_, NS = NS_;
    static constexpr int SLOTS = MK_WARPS / WPR;
    static constexpr int RC = SLOTS * RPW;
    static constexpr int RS = RC / NS;
    static constexpr int NB_MAX = 32 * WPR * BPL;
    static_assert(RC * WPR <= 64, "row partials fit rowred");
};
using MC0 = MCfg<1, 1, 2>;  // K <= 1024:  32 rows per chunk
using MC1 = MCfg<1, 2, 1>;  // K <= 2048:  16 rows
using MC2 = MCfg<2, 2, 1>;  // K <= 4096:   8 rows
using MC3 = MCfg<4, 2, 1>;  // K <= 8192:   4 rows
using MC4 = MCfg<8, 2, 1>;  // K <= 16384:  2 rows
using MD0 = MCfg<1, 1, 4, 2>;  // the same K ranges, two slots per chunk: 64 rows
using MD1 = MCfg<1, 2, 2, 2>;  // 32 rows
using MD2 = MCfg<2, 2, 2, 2>;  // 16 rows
using MD3 = MCfg<4, 2, 2, 2>;  //  8 rows
using MD4 = MCfg<8, 2, 2, 2>;  //  4 rows
constexpr int MK_NCFG = 5;     // configs 0-4 one slot per chunk, 5-9 two

inline int mk_cfg_for(int K) {
    const int nb = K / 32;
    if (nb <= MC0::NB_MAX) return 0;
    if (nb <= MC1::NB_MAX) return 1;
    if (nb <= MC2::NB_MAX) return 2;
    if (nb <= MC3::NB_MAX) return 3;
    if (nb <= MC4::NB_MAX) return 4;
    return -1;
}
inline int mk_rc(int cfg) {  // rows per chunk
    static const int rc[2 * MK_NCFG] = {MC0::RC, MC1::RC, MC2::RC, MC3::RC, MC4::RC,
                                        MD0::RC, MD1::RC, MD2::RC, MD3::RC, MD4::RC};
    return rc[cfg];
}
inline int mk_ns(int cfg) { return cfg >= MK_NCFG ? 2 : 1; }  // ring slots per chunk

enum { SK_GEMV = 0, SK_ATTN = 1, SK_FFN = 2, SK_OCOL = 3 };

// Fixed-point residual accumulators: the O-projection and FFN stages add
// their partial sums into int64 words scaled by 2^32 with integer atomics, so
// the totals do not depend on the order in which CTAs arrive.
constexpr float MK_FIX = 4294967296.0f;      // 2^32
constexpr float MK_UNFIX = 2.3283064365386963e-10f;  // 2^-32
constexpr int MK_DOWN_ROWS = MK_SLOT_PAY / 16;  // rows of one down-projection slot (1024)
__host__ __device__ __forceinline__ long long* acc_at(long long* a, int r) { return a + r; }

struct MStage {
    int kind, cfg, pro, epi;
    int K, N, RC, nchunks;
    // FFN: act blocks (units), gate/up chunks and down slots per unit.
    // OCOL: units (query head x RC-row chunk), ring slots per unit, column
    // blocks per slot.
    int nunits, per0, per1, N2;
    // PRO_NORM: the residual is base + racc (acc_in >= 1) + racc2 (acc_in ==
    // 2), added in that order; with post_a / post_f (post-norm families)
    // each accumulator is first rmsnorm'd with those unit gains.  nobar: the
    // stage starts without a grid barrier (its inputs are guarded by ready
    // counters).  window: ATTN / OCOL: sliding-window keys (0 = all).
    int acc_in, layer, nobar, window;
    long long* racc;
    long long* racc2;
    long long* acc_out;       // FFN / OCOL: the accumulator its partial sums are added into
    long long* zero_a;        // FFN: accumulators of the previous layer, zeroed here (this
    long long* zero_b;        //      CTA's slice of rows)
    const float* post_a;      // PRO_NORM: post-attention norm gains of racc (or null)
    const float* post_f;      // PRO_NORM: post-FFN norm gains of racc2 (or null)
    const void* pad_ptr;
    float* fold_to;        // QKV stage: this CTA's slice of the residual is stored here
    const float* base;     // PRO_NORM input (null: this CTA's embedding row)
    const float* norm_w;
    float* xn_out;         // CTA 0 stores the normalised input here
    float* y;
    const float* bias;
    // attention stage of one layer
    const float* q_norm;
    const float* k_norm;
    float* kc;             // this layer's K cache [n_kv][max_seq][hd]
    float* vc;
};
static_assert(sizeof(MStage) % 16 == 0, "stage descriptors are copied in 16-byte pieces");
static_assert(MK_DOWN_ROWS % MK_THREADS == 0, "whole rows per thread in one-block-per-row slots");
static_assert(MK_SLOTS >= 4, "a head's O-projection column blocks (head_dim <= 128) fit the ring");

// The weight-copy schedule of one stage (nchunks 0: no weights), kept in
// shared memory so the copy issuer never waits on a global read.  The
// matrices are the slot-packed copies the host builds for the step
// (cw_step.cu, k_pack_rows / k_pack_cols): every ring slot is filled by ONE
// bulk copy of a contiguous [payload | scales] range.
//   row slabs (pk0: GEMV weight, FFN gate/up): rows [s*rc, +rc) at byte
//     s*rc*nb*18, their payload (row-major, nb blocks of 16 B) then scales
//   column groups (pk1: FFN down with per1 == 1 column block per slot and
//     1024-row slabs; O projection with per1 column blocks per slot and
//     rc-row units): blocks [g*G, +G) over rows [r0, +rows) at byte
//     (g*dim + r0)*G*18, payload [block][row] then scales [block][row]
struct MIssue {
    const uint8_t* pk0;   // GEMV weight, or the FFN gate/up matrix (row slabs)
    const uint8_t* pk1;   // FFN down / O projection (column groups)
    int n0;               // GEMV: chunks; FFN: units (act blocks); OCOL: units
    int rc, nb, n;        // rows per copy (ring slot), blocks per row, rows of pk0
    int per0, per1;       // GEMV: slots per chunk; FFN: gate/up copies and down slots per unit
    int dim;              // FFN / OCOL: rows of pk1
    int kind;
    int pad[4];
};
static_assert(sizeof(MIssue) == 64, "issue entries are copied as four int4");

struct MParams {
    const MStage* stages;
    const MIssue* issues;
    int n_stages;
    DevState* st;
    int* status;
    unsigned long long* bar;
    const uint8_t* emb_payload;
    const __half* emb_scales;
    float embed_scale;
    float* hidden;
    // the QKV rows as 8-byte words: float bits | tag << 32, the tag naming the
    // (step, layer) that wrote them (mk_qkv_tag); the attention units poll the
    // words of their kv group until the tag is theirs, so the hand-off needs
    // no fence, counter or barrier
    unsigned long long* qkv;
    float* attn;
    const unsigned* prompt;
    unsigned* toks;
    float* part;
    unsigned* counters;
    const float* inv_freq;
    int dim, n_heads, n_kv, hd, max_seq, n_splits, part_stride, decode;
    int n_layers;
    int attn_min;  // keys per attention split before splitting further
    int window_next;  // window of the layer after a non-windowed one (alternating families)
    // Ready counters [n_layers][n_kv], zeroed at the end of every step: the
    // attention units of each kv head finished (the O-projection units wait
    // for the step's active split count).
    unsigned* ardy;
    long long* zero_a;  // the last layer's accumulators, zeroed at the end of the step
    long long* zero_b;
    float eps, scale;
    int unit;             // norm gains 1 + w (UnitShift) instead of w
    int geglu;            // FFN activation GeGLU (gelu_tanh) instead of SwiGLU
    float attn_softcap;   // attention logits cap * tanh(s / cap) (0 = off)
    float final_softcap;  // LM-head logits cap * tanh(l / cap) (0 = off)
    float inv_dim;      // 1/dim: the mean of squares as a product (exact for power-of-two dims)
    size_t work_bytes;  // shared-memory work region (q24 + hbuf + wbuf, or attention scratch)
    // profiling only: per stage and CTA, %globaltimer at the stage's start
    // (after its barrier), after its input prologue, after its main loop and
    // at the end of its work ([stage][cta][MK_STAMPS]; 0 = no work here)
    unsigned long long* stamps;
};

// Keys per warp iteration of the step's attention: ATTN_U, two for head_dim
// 256 (its K/V rows take twice the registers); a split is worth its combine
// from one iteration of all 16 warps on.
__host__ __device__ constexpr int mk_attn_u(int epl) { return epl >= 8 ? 2 : ATTN_U; }
__host__ __device__ constexpr int mk_attn_min(int epl) { return MK_WARPS * mk_attn_u(epl); }
// With 2..MK_DEFER active key splits, the attention stage only publishes each
// split's (accumulator, max, denominator) and the O-projection stage merges
// the splits of its head while it builds its input (no combine step, fence or
// counter inside the attention stage); with more splits the attention stage
// combines.
constexpr int MK_DEFER = 8;
// Floats per published split row (accumulator[hd], max, denominator, 2 pad):
// a multiple of four, so every row starts 16-byte aligned.
__host__ __device__ constexpr int mk_part_w(int hd) { return hd + 4; }

// per-CTA state shared by all threads
struct MShared {
    uint64_t full[MK_SLOTS];   // a slot's copy has landed
    uint64_t empty[MK_SLOTS];  // the compute warps are done with a slot
    uint64_t pol;  // L2 evict-first policy of the weight stream
    int issued, abort, last, prod_done;
    __align__(16) float act[32];  // FFN: the act block of the current unit
    __align__(16) uint4 aq[6];    // FFN: its q24 planes
    int acb;
    float asb;
    __align__(16) float red[2][MK_WARPS];  // CTA-sum partials, alternating per call
    unsigned long long keys[MK_WARPS];
    // RoPE angle pos * inv_freq[k] of this step's position: sin and cos,
    // computed once at the kernel start (every layer rotates at that position)
    float rsin[128], rcos[128];  // RoPE table of this position (head_dim <= 256)
};

struct MCtx {
    unsigned char* ring;
    unsigned char* work;
    float* emb;
    const MIssue* iss;  // shared-memory copy of the issue table
    float* rowred;      // 2 x 64 row partials
    MShared* sh;
    int seq;            // chunks consumed by this CTA so far (same in every thread)
    unsigned tag0;      // QKV word tag of layer 0 this step (mk_qkv_tag)
    int redsel;         // CTA-sum buffer of the next call
    int nch;            // chunks consumed (row-partial buffer parity)
    int pos;
    unsigned long long* stamp;  // this stage's stamps (profiling) or null
};

// CTA-wide sum with one CTA barrier: the warps' partials go to one of two
// alternating buffers, so a call never overwrites the buffer the previous
// call is still reading (every thread passed that call's barrier first).
// Fixed summation order.
__device__ __forceinline__ float mk_cta_sum(float v, MCtx& c) {
    static_assert(MK_WARPS == 16, "four float4 partial loads");
    v = warp_sum(v);
    float* r = c.sh->red[c.redsel];
    c.redsel ^= 1;
    if ((threadIdx.x & 31) == 0) r[threadIdx.x >> 5] = v;
    mk_sync();
    const float4* r4 = reinterpret_cast<const float4*>(r);
    const float4 a = r4[0], b = r4[1], d = r4[2], e = r4[3];
    return (((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w))) +
           (((d.x + d.y) + (d.z + d.w)) + ((e.x + e.y) + (e.z + e.w)));
}

// Lane 0 of the producer warp issues the weight copies.
constexpr int MK_ISSUER = MK_THREADS;

__device__ __forceinline__ void mk_clk(const MCtx& c, int k) {
    if (c.stamp && threadIdx.x == 0) c.stamp[4 + k] = clock64();
}

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int* p) {
    int v;
    asm volatile("ld.volatile.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(unsigned long long* p, unsigned long long v) {
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// The producer lane: fill the next ring slot with `bytes` (a multiple of 16)
// from the contiguous packed range at src, in one bulk copy.
__device__ __forceinline__ void mk_issue_copy(MShared* sh, unsigned char* ring, const uint8_t* src,
                                              unsigned bytes) {
    const int slot = sh->issued % MK_SLOTS;
    unsigned char* dst = ring + (size_t)slot * MK_SLOT_BYTES;
    // the slot's previous contents were read before the compute warps'
    // release of it (its "empty" mbarrier, which the producer waited on): a
    // generic-proxy read followed by an async-proxy write, ordered by that
    // mbarrier, no proxy fence
    mbar_expect_tx(&sh->full[slot], bytes);  // 0: a plain arrive (rows past the end)
    if (bytes) bulk_g2s_hint(dst, src, bytes, &sh->full[slot], sh->pol);
    sh->issued++;
}

// A position in this CTA's sequence of weight copies (the stage order of
// the issue table).
struct MIter {
    int stage, t, j;
};

// The copy after position it (its packed source range; bytes 0: rows past
// the end of a matrix, an empty slot) and advance it.  False when the step
// has no more copies.  Out of line: only the producer lane runs it.
static __device__ __noinline__ bool mk_next_copy(const MIssue* iss, int n_stages, MIter& it,
                                                 const uint8_t** src, unsigned* bytes) {
    while (it.stage < n_stages) {
        const MIssue& I = iss[it.stage];
        const long u = blockIdx.x + (long)it.t * gridDim.x;
        if (I.kind == SK_GEMV) {  // copy t: part t % per0 of this CTA's chunk t / per0
            const long ch = blockIdx.x + (long)(it.t / I.per0) * gridDim.x;
            if (ch < I.n0) {
                const long row0 = (ch * I.per0 + it.t % I.per0) * I.rc;
                const int rows = (int)max(0L, min((long)I.rc, (long)I.n - row0));
                *src = I.pk0 + (size_t)row0 * I.nb * 18;
                *bytes = (unsigned)rows * I.nb * 18;
                it.t++;
                return true;
            }
        }
        if (I.kind == SK_OCOL && u < I.n0) {
            // unit u = (query head h, rows [r0, r0 + rc)); ring slot j of the
            // unit holds column group h*per0 + j (column blocks
            // h*nb + j*per1 .. + per1 - 1) over those rows
            const int nch = (I.dim + I.rc - 1) / I.rc, h = (int)(u / nch);
            const int r0 = (int)(u - (long)h * nch) * I.rc, rows = min(I.rc, I.dim - r0);
            const size_t g = (size_t)h * I.per0 + it.j;
            *src = I.pk1 + (g * I.dim + r0) * I.per1 * 18;
            *bytes = (unsigned)(I.per1 * rows * 18);
            if (++it.j == I.per0) {
                it.j = 0;
                it.t++;
            }
            return true;
        }
        if (I.kind == SK_FFN && u < I.n0) {
            if (it.j < I.per0) {  // gate/up rows [64u + j*rc, +rc)
                const long row0 = u * 64 + (long)it.j * I.rc;
                *src = I.pk0 + (size_t)row0 * I.nb * 18;
                *bytes = (unsigned)I.rc * I.nb * 18;
            } else {  // down rows [k*1024, ...) of column block u
                const int k = it.j - I.per0, r0 = k * MK_DOWN_ROWS;
                const int rows = min(MK_DOWN_ROWS, I.dim - r0);
                *src = I.pk1 + ((size_t)u * I.dim + r0) * 18;
                *bytes = (unsigned)rows * 18;
            }
            if (++it.j == I.per0 + I.per1) {
                it.j = 0;
                it.t++;
            }
            return true;
        }
        it.stage++;
        it.t = 0;
        it.j = 0;
    }
    return false;
}

// Compute thread 0, after the CTA barrier that ends the use of ring slots
// seq .. seq+n-1: hand them back to the producer.
__device__ __forceinline__ void mk_release(MCtx& c, int n) {
    if (threadIdx.x == 0)
        for (int k = 0; k < n; k++)
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(
                             smem_addr(&c.sh->empty[(c.seq + k) % MK_SLOTS]))
                         : "memory");
}

__device__ __forceinline__ int ld_volatile_shared_i32(const int* p) {
    return *reinterpret_cast<const volatile int*>(p);
}

// The producer warp's lane 0: queue every weight copy of the step in order,
// copy q into ring slot q % MK_SLOTS once the compute warps released that
// slot's previous copy (q - MK_SLOTS).  Stops early when the CTA aborts.
// (An L2 prefetch of the copies one ring ahead made the step slower: 0.64 ->
// 0.67 ms/token at Qwen3-0.6B, 2.36 -> 2.76 at Qwen3-8B.)
__device__ inline void mk_produce(const MParams& p, MCtx& c) {
    MShared* sh = c.sh;
    MIter it = {0, 0, 0};
    for (int q = 0;; q++) {
        if (q >= MK_SLOTS) {
            uint64_t* e = &sh->empty[q % MK_SLOTS];
            const unsigned par = (unsigned)(((q / MK_SLOTS) - 1) & 1);
            bool ok = mbar_try_wait(e, par);
            const uint64_t t0 = ok ? 0 : global_ns();
            while (!ok) {
                if (ld_volatile_shared_i32(&sh->abort)) break;
                if (global_ns() - t0 > MK_WAIT_NS) {
                    atomicExch(p.status, (int)DEV_TIMEOUT);
                    sh->abort = 1;
                    break;
                }
                ok = mbar_try_wait(e, par);
            }
            if (!ok) break;
        }
        const uint8_t* src;
        unsigned bytes;
        if (ld_volatile_shared_i32(&sh->abort) || !mk_next_copy(c.iss, p.n_stages, it, &src, &bytes))
            break;
        mk_issue_copy(sh, c.ring, src, bytes);
    }
    __threadfence_block();
    *reinterpret_cast<volatile int*>(&sh->prod_done) = 1;
}

// Compute threads: wait (bounded) until the producer has stopped, then for
// every copy issued and not yet consumed, so no bulk copy writes shared
// memory after the CTA has left.
__device__ inline void mk_drain(MCtx& c) {
    if (threadIdx.x == 0) {
        const uint64_t t0 = global_ns();
        while (!ld_volatile_shared_i32(&c.sh->prod_done) && global_ns() - t0 < MK_WAIT_NS) {
        }
        const int issued = ld_volatile_shared_i32(&c.sh->issued);
        for (int q = c.seq; q < issued; q++)
            mbar_wait(&c.sh->full[q % MK_SLOTS], (unsigned)((q / MK_SLOTS) & 1), MK_WAIT_NS);
    }
    mk_sync();
}

__device__ inline void mk_fail(const MParams& p, MCtx& c) {
    if (threadIdx.x == 0) {
        atomicExch(p.status, (int)DEV_TIMEOUT);
        *reinterpret_cast<volatile int*>(&c.sh->abort) = 1;
    }
    mk_sync();
}

// Grid-wide barrier: a CTA barrier orders the compute warps' writes before
// thread 0's gpu-scope release arrive; thread 0 polls (acquire) until the
// counter reaches `target`, and a CTA barrier passes that on.  The status
// word and the time limit are checked every 64 polls.
__device__ inline bool mk_grid_sync(const MParams& p, MCtx& c, unsigned long long target,
                                    uint64_t limit_ns = MK_WAIT_NS) {
    mk_sync();  // the compute warps' writes before thread 0's release arrive
    if (threadIdx.x == 0) {
        red_release_add(p.bar, 1ull);
        uint64_t t0 = 0;
        int ok = 1;
        for (unsigned it = 1; ld_acquire_u64(p.bar) < target; it++) {
            if ((it & 63) == 0) {
                const uint64_t now = global_ns();
                if (t0 == 0) t0 = now;
                if (ld_volatile_i32(p.status) != 0 || now - t0 > limit_ns) {
                    ok = 0;
                    break;
                }
            }
        }
        if (!ok) {
            atomicExch(p.status, (int)DEV_TIMEOUT);
            *reinterpret_cast<volatile int*>(&c.sh->abort) = 1;
        }
    }
    mk_sync();
    return c.sh->abort == 0;
}

// One thread: bounded wait until the ready counter reaches `target` (acquire:
// the producers' stores before their release add are visible afterwards).
// A timeout, or an error raised by another CTA, sets the status word and the
// CTA's abort flag.
__device__ inline bool mk_wait_count(const MParams& p, MCtx& c, const unsigned* ctr,
                                     unsigned target) {
    uint64_t t0 = 0;
    for (unsigned it = 1; ld_acquire_u32(ctr) < target; it++) {
        if ((it & 63) == 0) {
            const uint64_t now = global_ns();
            if (t0 == 0) t0 = now;
            if (ld_volatile_i32(p.status) != 0 || now - t0 > MK_WAIT_NS) {
                atomicExch(p.status, (int)DEV_TIMEOUT);
                *reinterpret_cast<volatile int*>(&c.sh->abort) = 1;
                return false;
            }
        }
    }
    return true;
}

// Rows per CTA of the residual slices the QKV stage stores (fold_to) and the
// FFN stage zeroes: a multiple of four, so slices are float4 groups.
__device__ __forceinline__ int mk_slice_rows(int dim) {
    return (((dim + gridDim.x - 1) / gridDim.x) + 3) & ~3;
}

// Stage descriptors travel global -> shared by cp.async (16 bytes per thread
// of the loader lanes, no register staging), requested two stages ahead and
// waited for at the end of the current stage, so no thread ever stalls on
// the descriptor table.
constexpr int MK_LOADER = MK_THREADS - 32;  // first thread of the loader lanes (last warp)
static_assert(sizeof(MStage) / 16 <= 32, "one 16-byte piece per loader lane");
__device__ __forceinline__ void mk_load_stage(const MParams& p, int si, MStage* dst) {
    const int l = threadIdx.x - MK_LOADER;
    if (si < p.n_stages && l >= 0 && l < (int)(sizeof(MStage) / 16)) {
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                         smem_addr(reinterpret_cast<char*>(dst) + 16 * l)),
                     "l"(reinterpret_cast<const char*>(p.stages + si) + 16 * l)
                     : "memory");
        asm volatile("cp.async.commit_group;" ::: "memory");
    }
}
__device__ __forceinline__ void mk_load_stage_wait() {
    if (threadIdx.x >= MK_LOADER) asm volatile("cp.async.wait_all;" ::: "memory");
}

// ---- stage input -> q24 planes ---------------------------------------------------
// Four consecutive elements per lane: lane L of a warp covers block
// 4t + L/8 (t: the warp's quad group), elements 4*(L%8) .. 4*(L%8)+3, loaded
// as one float4.  The block max and the integer sum are 3-step shuffles
// within the 8 lanes of a block, and each lane writes one 32-bit word per
// byte plane (its 4 elements' bytes, packed with __byte_perm) -- the planes
// q24_block writes, in a quarter of the instructions.
constexpr int MK_QB = 2;  // quad groups per warp per batch

__device__ __forceinline__ void mk_q24_quad(const Q24& s, int b, bool valid, const float4& v,
                                            int lane) {
    q24_quad(s, b, valid, v, lane);
}

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
// h + 2^-32 * (accumulator rows i .. i+3; i % 4 == 0)
__device__ __forceinline__ float4 mk_add_fixed4(float4 h, const long long* acc, int i) {
    const longlong2 a0 = __ldcg(reinterpret_cast<const longlong2*>(acc + i));
    const longlong2 a1 = __ldcg(reinterpret_cast<const longlong2*>(acc + i + 2));
    h.x = h.x + __ll2float_rn(a0.x) * MK_UNFIX;
    h.y = h.y + __ll2float_rn(a0.y) * MK_UNFIX;
    h.z = h.z + __ll2float_rn(a1.x) * MK_UNFIX;
    h.w = h.w + __ll2float_rn(a1.y) * MK_UNFIX;
    return h;
}
__device__ __forceinline__ float4 f4_norm(const float4& h, float inv, const float4& g) {
    return make_float4(__fmul_rn(__fmul_rn(h.x, inv), g.x), __fmul_rn(__fmul_rn(h.y, inv), g.y),
                       __fmul_rn(__fmul_rn(h.z, inv), g.z), __fmul_rn(__fmul_rn(h.w, inv), g.w));
}

// Elements d0 .. d0+3 of query head h's attention output.  With 2..MK_DEFER
// active splits: the merge of the splits' published states
// (attention.wgsl:88-95 across splits: M = max_s m_s, c_s = exp(m_s - M),
// L = sum_s l_s c_s, x = (sum_s acc_s c_s) / L), from split rows of
// mk_part_w(hd) floats (16-byte aligned), so the four accumulator values and
// the (m_s, l_s) pair of every split come in ONE round of L2 loads.  Else
// the normalised output the attention stage wrote to p.attn.
static __device__ __noinline__ float4 mk_head_out4(const float* attn, const float* part, int part_stride,
                                            int hd, int h, int d0, int na) {
    if (na < 2 || na > MK_DEFER)
        return __ldcg(reinterpret_cast<const float4*>(attn + (size_t)h * hd + d0));
    const int WP = mk_part_w(hd);
    const float* ph = part + (size_t)h * part_stride * WP;
    float4 pv[MK_DEFER];
    float2 ml[MK_DEFER];
#pragma unroll
    for (int s = 0; s < MK_DEFER; s++) {
        pv[s] = s < na ? __ldcg(reinterpret_cast<const float4*>(ph + (size_t)s * WP + d0))
                       : make_float4(0.f, 0.f, 0.f, 0.f);
        ml[s] = s < na ? __ldcg(reinterpret_cast<const float2*>(ph + (size_t)s * WP + hd))
                       : make_float2(REF_NEG_INF, 0.f);
    }
    float M = ml[0].x;
#pragma unroll
    for (int s = 1; s < MK_DEFER; s++) M = s < na ? fmaxf(M, ml[s].x) : M;
    float cc[MK_DEFER], L = 0.f;
#pragma unroll
    for (int s = 0; s < MK_DEFER; s++) {
        cc[s] = s < na ? expf(ml[s].x - M) : 0.f;
        L = s < na ? fmaf(ml[s].y, cc[s], L) : L;
    }
    // splits in groups of four, fixed summation tree
    float r[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s0 = 0; s0 < MK_DEFER; s0 += 4) {
        float a[4][4];
#pragma unroll
        for (int j = 0; j < 4; j++) {
            a[j][0] = pv[s0 + j].x * cc[s0 + j];
            a[j][1] = pv[s0 + j].y * cc[s0 + j];
            a[j][2] = pv[s0 + j].z * cc[s0 + j];
            a[j][3] = pv[s0 + j].w * cc[s0 + j];
        }
#pragma unroll
        for (int e = 0; e < 4; e++)
            if (s0 < na) r[e] = r[e] + ((a[0][e] + a[1][e]) + (a[2][e] + a[3][e]));
    }
    const float inv = 1.0f / L;
    return make_float4(r[0] * inv, r[1] * inv, r[2] * inv, r[3] * inv);
}

// The stage input as q24 planes: the rmsnorm of `base` (plus the fixed-point
// accumulators acc_in names) with the gains (norm.wgsl:20-56).  Each batch
// issues all of its global loads before using any.  Inputs of up to
// 4 * MK_WARPS * MK_QB blocks (K <= 4096) are one batch held in registers;
// BIG kernels (K up to 16384) also compile the staged multi-batch path.
template <class LD>
__device__ inline void mk_prologue_staged(const MParams& p, const MStage& S, const Q24& q,
                                          float* hbuf, float* wbuf, MCtx& c, const LD& ld_src);
__device__ inline void mk_prologue_tail(const MParams& p, const MStage& S, const Q24& q, MCtx& c,
                                        float4 (&v)[MK_QB]);
// h * 2^-32 for the four accumulator rows i .. i+3
__device__ __forceinline__ float4 mk_fixed4(const long long* acc, int i) {
    return mk_add_fixed4(f4_zero(), acc, i);
}
__device__ __forceinline__ float4 f4_add(const float4& a, const float4& b) {
    return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}
__device__ __forceinline__ float4 f4_unit(const float4& w) {  // 1 + w (UnitShift gains)
    return make_float4(1.0f + w.x, 1.0f + w.y, 1.0f + w.z, 1.0f + w.w);
}
__device__ __forceinline__ float f4_ss(const float4& v, float ss) {
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    return fmaf(v.w, v.w, ss);
}

// POST (post-norm families, Gemma-2): the residual is
// base + rmsnorm_unit(racc; post_a) + rmsnorm_unit(racc2; post_f), the
// additions of the reference composition's x = x + post_norm(o) and
// x = x + post_norm(ffn) (one batch in registers: K <= 4096).
template <bool BIG, bool POST>
__device__ inline void mk_prologue(const MParams& p, const MStage& S, const Q24& q, float* hbuf,
                            float* wbuf, MCtx& c) {
    const int nb = S.K / 32, nq = nb / 4;  // quad groups (nb is a multiple of 8)
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane >> 3, e0 = 4 * (lane & 7);
    const float* src = S.base ? S.base : c.emb;
    const bool gsrc = S.base != nullptr;
    // the residual: base (+ the fixed-point FFN accumulator when acc_in)
    auto ld_src = [&](int i) {
        float4 h = gsrc ? __ldcg(reinterpret_cast<const float4*>(src + i))
                        : *reinterpret_cast<const float4*>(src + i);
        if (S.acc_in >= 1) h = mk_add_fixed4(h, S.racc, i);
        if (S.acc_in >= 2) h = mk_add_fixed4(h, S.racc2, i);
        return h;
    };
    if constexpr (POST) {
        static_assert(!BIG, "post-norm residuals are formed in one batch");
        float4 v[MK_QB], ya[MK_QB], zf[MK_QB], ga[MK_QB], gf[MK_QB];
        float ssa = 0.f, ssf = 0.f;
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {
            const int b = 4 * (warp + k * MK_WARPS) + sub, i = b * 32 + e0;
            const bool in = b < nb;
            v[k] = !in ? f4_zero()
                       : gsrc ? __ldcg(reinterpret_cast<const float4*>(src + i))
                              : *reinterpret_cast<const float4*>(src + i);
            ya[k] = in && S.acc_in >= 1 ? mk_fixed4(S.racc, i) : f4_zero();
            zf[k] = in && S.acc_in >= 2 ? mk_fixed4(S.racc2, i) : f4_zero();
            ga[k] = in && S.acc_in >= 1 ? __ldg(reinterpret_cast<const float4*>(S.post_a + i)) : f4_zero();
            gf[k] = in && S.acc_in >= 2 ? __ldg(reinterpret_cast<const float4*>(S.post_f + i)) : f4_zero();
            ssa = f4_ss(ya[k], ssa);
            ssf = f4_ss(zf[k], ssf);
        }
        if (S.acc_in >= 1) {
            const float inva = 1.0f / sqrtf(mk_cta_sum(ssa, c) * p.inv_dim + p.eps);
#pragma unroll
            for (int k = 0; k < MK_QB; k++) v[k] = f4_add(v[k], f4_norm(ya[k], inva, f4_unit(ga[k])));
        }
        if (S.acc_in >= 2) {
            const float invf = 1.0f / sqrtf(mk_cta_sum(ssf, c) * p.inv_dim + p.eps);
#pragma unroll
            for (int k = 0; k < MK_QB; k++) v[k] = f4_add(v[k], f4_norm(zf[k], invf, f4_unit(gf[k])));
        }
        mk_prologue_tail(p, S, q, c, v);
        return;
    }
    if (!BIG || nq <= MK_WARPS * MK_QB) {  // one batch: everything stays in registers
        float4 v[MK_QB];
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {
            const int b = 4 * (warp + k * MK_WARPS) + sub, i = b * 32 + e0;
            v[k] = b < nb ? ld_src(i) : f4_zero();
        }
        mk_prologue_tail(p, S, q, c, v);
        return;
    }
    if constexpr (BIG) mk_prologue_staged(p, S, q, hbuf, wbuf, c, ld_src);
}

// One-batch prologue from the residual v (four elements per lane per
// quad group): this CTA's fold slice, the CTA-wide rmsnorm, the q24 planes.
__device__ inline void mk_prologue_tail(const MParams& p, const MStage& S, const Q24& q, MCtx& c,
                                        float4 (&v)[MK_QB]) {
    const int nb = S.K / 32, nq = nb / 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane >> 3, e0 = 4 * (lane & 7);
    const bool wx = S.xn_out && blockIdx.x == 0;
    float ss = 0.f;
    {
        float4 w[MK_QB];
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {
            const int b = 4 * (warp + k * MK_WARPS) + sub, i = b * 32 + e0;
            w[k] = b < nb ? __ldg(reinterpret_cast<const float4*>(S.norm_w + i)) : f4_zero();
            if (p.unit) w[k] = f4_unit(w[k]);
        }
        if (S.fold_to) {  // this CTA's slice of the residual: the next stages' base
            const int rs = mk_slice_rows(S.K), lo = blockIdx.x * rs;
#pragma unroll
            for (int k = 0; k < MK_QB; k++) {
                const int b = 4 * (warp + k * MK_WARPS) + sub, i = b * 32 + e0;
                if (b < nb && i >= lo && i < lo + rs)
                    *reinterpret_cast<float4*>(S.fold_to + i) = v[k];
            }
        }
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {  // padding adds +0
            ss = fmaf(v[k].x, v[k].x, ss);
            ss = fmaf(v[k].y, v[k].y, ss);
            ss = fmaf(v[k].z, v[k].z, ss);
            ss = fmaf(v[k].w, v[k].w, ss);
        }
        mk_clk(c, CLK_LOADED);
        ss = mk_cta_sum(ss, c);
        mk_clk(c, CLK_NORMED);
        const float inv = 1.0f / sqrtf(ss * p.inv_dim + p.eps);
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {
            const int b = 4 * (warp + k * MK_WARPS) + sub;
            v[k] = f4_norm(v[k], inv, w[k]);
            if (wx && b < nb) *reinterpret_cast<float4*>(S.xn_out + b * 32 + e0) = v[k];
        }
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {
            const int b = 4 * (warp + k * MK_WARPS) + sub;
            if (warp + k * MK_WARPS < nq) mk_q24_quad(q, b, b < nb, v[k], lane);
        }
    }
}

// The multi-batch path of mk_prologue: inputs staged in shared memory.
template <class LD>
__device__ inline void mk_prologue_staged(const MParams& p, const MStage& S, const Q24& q,
                                          float* hbuf, float* wbuf, MCtx& c, const LD& ld_src) {
    const int nb = S.K / 32, nq = nb / 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = lane >> 3, e0 = 4 * (lane & 7);
    const bool wx = S.xn_out && blockIdx.x == 0;
    float ss = 0.f;
    for (int t0 = warp; t0 < nq; t0 += MK_WARPS * MK_QB) {
        float4 v[MK_QB], w[MK_QB];
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {
            const int b = 4 * (t0 + k * MK_WARPS) + sub, i = b * 32 + e0;
            v[k] = b < nb ? ld_src(i) : f4_zero();
            w[k] = b < nb ? __ldg(reinterpret_cast<const float4*>(S.norm_w + i)) : f4_zero();
            if (p.unit) w[k] = f4_unit(w[k]);
        }
#pragma unroll
        for (int k = 0; k < MK_QB; k++) {
            const int b = 4 * (t0 + k * MK_WARPS) + sub, i = b * 32 + e0;
            if (b < nb) {
                *reinterpret_cast<float4*>(hbuf + i) = v[k];
                *reinterpret_cast<float4*>(wbuf + i) = w[k];
            }
            ss = fmaf(v[k].x, v[k].x, ss);
            ss = fmaf(v[k].y, v[k].y, ss);
            ss = fmaf(v[k].z, v[k].z, ss);
            ss = fmaf(v[k].w, v[k].w, ss);
        }
    }
    mk_clk(c, CLK_LOADED);
    ss = mk_cta_sum(ss, c);  // its barrier also publishes hbuf
    mk_clk(c, CLK_NORMED);
    if (S.fold_to) {  // this CTA's slice of the residual: the next stages' base
        const int rs = mk_slice_rows(S.K), i = blockIdx.x * rs + 4 * threadIdx.x;
        if (4 * (int)threadIdx.x < rs && i < S.K)
            *reinterpret_cast<float4*>(S.fold_to + i) = *reinterpret_cast<const float4*>(hbuf + i);
    }
    const float inv = 1.0f / sqrtf(ss * p.inv_dim + p.eps);
    for (int t = warp; t < nq; t += MK_WARPS) {
        const int b = 4 * t + sub, i = b * 32 + e0;
        float4 v = f4_zero();
        if (b < nb) {
            v = f4_norm(*reinterpret_cast<const float4*>(hbuf + i), inv,
                        *reinterpret_cast<const float4*>(wbuf + i));
            if (wx) *reinterpret_cast<float4*>(S.xn_out + i) = v;
        }
        mk_q24_quad(q, b, b < nb, v, lane);
    }
}

// ---- GEMV stage ------------------------------------------------------------------
// T = sum_j (q_j - 8) X_j of one Q4_0 block (16 payload bytes w) against one
// q24 block (planes xa: elements 0-15, xb: 16-31; cb = 8 * sum X): six
// independent dp4a chains of four, low and high nibbles apart.
__device__ __forceinline__ float mk_block_dot(const uint4& w4, const uint4 (&xa)[3],
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
    for (int e = 0; e < 4; e++) {
        const unsigned lo = w[e] & 0x0f0f0f0fu;
        const unsigned hi = (w[e] >> 4) & 0x0f0f0f0fu;
        s0l = dp4a_uu(lo, a0[e], s0l);
        s0h = dp4a_uu(hi, b0[e], s0h);
        s1l = dp4a_uu(lo, a1[e], s1l);
        s1h = dp4a_uu(hi, b1[e], s1h);
        s2l = dp4a_us(lo, a2[e], s2l);
        s2h = dp4a_us(hi, b2[e], s2h);
    }
    const int s01 = (s0l + s0h) + ((s1l + s1h) << 8) - cb;
    return fmaf((float)(s2l + s2h), 65536.0f, (float)s01);
}

// The input vector of a GEMV stage as q24 planes in the work region.
constexpr int MK_ONE_BATCH_BLOCKS = 4 * MK_WARPS * MK_QB;
template <class CF, bool POST>
__device__ __forceinline__ void mk_input(const MParams& p, const MStage& S, const Q24& q,
                                         MCtx& c) {
    float* hbuf = reinterpret_cast<float*>(c.work + al16(q24_bytes(q.nb)));
    float* wbuf = hbuf + S.K;
    mk_prologue<(CF::NB_MAX > MK_ONE_BATCH_BLOCKS), POST>(p, S, q, hbuf, wbuf, c);
}

// This lane's blocks of the q24 planes, kept in registers for the chunk loop.
template <class CF>
struct MRegs {
    uint4 xa[CF::BPL][3], xb[CF::BPL][3];
    int cb[CF::BPL];
    float sb[CF::BPL];
};
template <class CF>
__device__ __forceinline__ void mk_load_regs(const Q24& q, MRegs<CF>& R) {
    constexpr int WPR = CF::WPR, BPL = CF::BPL;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wsub = warp % WPR;
#pragma unroll
    for (int k = 0; k < BPL; k++) {
        const int b = wsub * 32 + lane + k * 32 * WPR;
        const bool in = b < q.nb;
#pragma unroll
        for (int pl = 0; pl < 3; pl++) {
            R.xa[k][pl] = in ? q.pl[(pl * 2 + 0) * q.nb + b] : make_uint4(0, 0, 0, 0);
            R.xb[k][pl] = in ? q.pl[(pl * 2 + 1) * q.nb + b] : make_uint4(0, 0, 0, 0);
        }
        R.cb[k] = in ? q.cb[b] : 0;
        R.sb[k] = in ? q.sb[b] : 0.f;
    }
}

// One chunk of RC rows: wait for ring slot c.seq, dot each row with the
// planes in R, reduce the per-warp partials into rb[row * WPR + sub], then
// (after the CTA barrier) hand the slots back to the producer.  Returns
// rb, or null after a timed-out wait (the failure is recorded).  Each thread
// waits on the slot's mbarrier itself, so the only CTA barrier is the one at
// the end: warps start on a chunk while the issuing lane is still queueing
// the copies of the previous one, and a failed wait (whose thread reads
// stale slot bytes, in bounds) is agreed on at that barrier.
template <class CF>
__device__ __forceinline__ const float* mk_chunk(const MParams& p, MCtx& c, int nb, int rows,
                                                 const MRegs<CF>& R, bool first) {
    constexpr int WPR = CF::WPR, BPL = CF::BPL, RPW = CF::RPW, NS = CF::NS, RS = CF::RS;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int wsub = warp % WPR, slot = warp / WPR;
    bool ok = true;
#pragma unroll
    for (int h = 0; h < NS; h++) {
        const int q = c.seq + h;
        ok = mbar_wait(&c.sh->full[q % MK_SLOTS], (unsigned)((q / MK_SLOTS) & 1), MK_WAIT_NS) && ok;
    }
    if (first) mk_clk(c, CLK_WAITED);
    // this warp's rows lie in one slot (RS is a multiple of RPW); the slot
    // holds min(RS, rows - h*RS) rows' payload, then their scales
    const int h = (slot * RPW) / RS;
    const unsigned char* pay = c.ring + (size_t)((c.seq + h) % MK_SLOTS) * MK_SLOT_BYTES;
    const int srows = max(0, min(RS, rows - h * RS));
    const __half* scs = reinterpret_cast<const __half*>(pay + (size_t)srows * nb * 16);
    float* rb = c.rowred + (size_t)(c.nch & 1) * 64;
    uint4 w4[RPW][BPL];
    float dd[RPW][BPL];
#pragma unroll
    for (int j = 0; j < RPW; j++) {
        const int r = slot * RPW + j, rr = r - h * RS;
#pragma unroll
        for (int k = 0; k < BPL; k++) {
            const int b = wsub * 32 + lane + k * 32 * WPR;
            const bool in = r < rows && b < nb;
            const size_t blk = in ? (size_t)rr * nb + b : 0;
            w4[j][k] = in ? reinterpret_cast<const uint4*>(pay)[blk] : make_uint4(0, 0, 0, 0);
            dd[j][k] = in ? __half2float(scs[blk]) : 0.f;
        }
    }
    float acc[RPW];
#pragma unroll
    for (int j = 0; j < RPW; j++) {
        acc[j] = 0.f;
#pragma unroll
        for (int k = 0; k < BPL; k++)
            acc[j] = fmaf(dd[j][k] * R.sb[k], mk_block_dot(w4[j][k], R.xa[k], R.xb[k], R.cb[k]),
                          acc[j]);
    }
    const float v = warp_reduce_rows<RPW>(acc, lane);
    if ((lane & (32 / RPW - 1)) == 0) rb[(slot * RPW + lane / (32 / RPW)) * WPR + wsub] = v;
    if (mk_sync_or(!ok)) {  // slots consumed, row partials complete
        mk_fail(p, c);
        return nullptr;
    }
    if (first) mk_clk(c, CLK_SUMMED);
    mk_release(c, NS);
    if (first) mk_clk(c, CLK_ISSUED);
    c.seq += NS;
    c.nch++;
    return rb;
}

// GEMV stage over the rmsnorm of the residual: EPI_STORE (the QKV
// projection, + bias) or EPI_HEAD (the LM head: logits and the argmax key).
// Each variant compiles only its own epilogue: the step kernel's code is
// streamed through the instruction caches once per layer, so what a stage
// does not run should not sit in its instruction stream.
template <class CF, int EPI, bool POST>
__device__ inline bool mk_gemv(const MParams& p, const MStage& S, MCtx& c) {
    static_assert(EPI == EPI_STORE || EPI == EPI_HEAD, "QKV or LM head");
    constexpr int WPR = CF::WPR, RC = CF::RC;
    const int nb = S.K / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if ((int)blockIdx.x >= S.nchunks) {  // no rows of this stage here
        if (POST && S.fold_to) {
            // but still this CTA's slice of the next residual base, which
            // takes the norms of the whole accumulators: the full prologue
            if ((int)blockIdx.x * mk_slice_rows(S.K) < S.K)
                mk_input<CF, POST>(p, S, q24_carve(c.work, nb), c);
        } else if (S.fold_to) {  // but still this CTA's slice of the next residual base
            const int rs = mk_slice_rows(S.K), i = blockIdx.x * rs + 4 * tid;
            if (4 * tid < rs && i < S.K) {
                float4 h = S.base ? __ldcg(reinterpret_cast<const float4*>(S.base + i))
                                  : *reinterpret_cast<const float4*>(c.emb + i);
                if (S.acc_in >= 1) h = mk_add_fixed4(h, S.racc, i);
                if (S.acc_in >= 2) h = mk_add_fixed4(h, S.racc2, i);
                *reinterpret_cast<float4*>(S.fold_to + i) = h;
            }
        }
        return true;
    }
    // the bias of the first chunk's rows, requested now so it arrives while
    // the prologue runs
    float add = 0.f;
    if (EPI == EPI_STORE && S.bias && tid < RC && (long)blockIdx.x * RC + tid < S.N)
        add = __ldg(S.bias + (long)blockIdx.x * RC + tid);
    const Q24 q = q24_carve(c.work, nb);
    mk_input<CF, POST>(p, S, q, c);
    mk_clk(c, CLK_Q24);
    mk_sync();
    MRegs<CF> R;
    mk_load_regs<CF>(q, R);
    if (c.stamp && tid == 0) c.stamp[1] = global_ns();
    mk_clk(c, CLK_REGS);
    unsigned long long best = argmax_key_init();
    int t = 0;
    for (long chunk = blockIdx.x; chunk < S.nchunks; chunk += gridDim.x, t++) {
        const long row0 = chunk * RC;
        const int rows = (int)min((long)RC, (long)S.N - row0);
        if (EPI == EPI_STORE && t > 0 && S.bias && tid < rows)  // requested before the wait
            add = __ldg(S.bias + row0 + tid);
        const float* rb = mk_chunk<CF>(p, c, nb, rows, R, t == 0);
        if (!rb) return false;
        // epilogue: fixed-order sum of the WPR partials of each row
        if (tid < rows) {
            float vv = 0.f;
#pragma unroll
            for (int w = 0; w < WPR; w++) vv += rb[tid * WPR + w];
            const long row = row0 + tid;
            if (EPI == EPI_HEAD) {
                if (p.final_softcap > 0.f) vv = p.final_softcap * tanhf(vv / p.final_softcap);
                S.y[row] = vv;
                const unsigned long long kk = argmax_key(vv, (unsigned)row);
                best = kk > best ? kk : best;
            } else {  // one tagged word per row (the attention units poll it)
                const float v = S.bias ? vv + add : vv;
                st_relaxed_u64(p.qkv + row, ((unsigned long long)(c.tag0 + S.layer) << 32) |
                                                __float_as_uint(v));
            }
        }
    }
    if (c.stamp && tid == 0) c.stamp[2] = global_ns();
    mk_clk(c, CLK_MAIN);
    if (EPI == EPI_HEAD) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long tt = __shfl_xor_sync(FULL, best, o);
            best = tt > best ? tt : best;
        }
        if (lane == 0) c.sh->keys[warp] = best;
        mk_sync();
        if (tid == 0) {
            for (int w = 1; w < MK_WARPS; w++) best = c.sh->keys[w] > best ? c.sh->keys[w] : best;
            atomicMax(&p.st->key, best);
        }
    }
    return true;
}

// ---- FFN stage: gate/up + SwiGLU + down projection, one act block per unit --------
// Unit u owns act block u (act rows 32u .. 32u+31 = gate/up rows 64u ..
// 64u+63, glu.wgsl:25): its gate/up chunks give the 32 act values, which are
// converted to one q24 block, and the down projection's column block u
// (MK_DOWN_ROWS rows per ring slot, one Q4_0 block per row) turns them into a
// partial sum for every output row, added into the fixed-point residual
// accumulator S.acc_out (the next stage that reads the residual adds it).
template <class CF, bool POST>
__device__ inline bool mk_ffn(const MParams& p, const MStage& S, MCtx& c) {
    constexpr int WPR = CF::WPR, RC = CF::RC;
    const int nb = S.K / 32;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (S.zero_a && warp == MK_WARPS - 1) {
        // the previous layer's accumulators: every reader (the QKV stage's
        // prologue) is behind this stage's barrier; zero this CTA's slice
        const int rs = mk_slice_rows(p.dim);
        for (int r = blockIdx.x * rs + lane; r < min((int)(blockIdx.x + 1) * rs, p.dim); r += 32) {
            *acc_at(S.zero_a, r) = 0;
            *acc_at(S.zero_b, r) = 0;
        }
    }
    if ((int)blockIdx.x >= S.nunits) return true;
    const Q24 q = q24_carve(c.work, nb);
    mk_input<CF, POST>(p, S, q, c);
    mk_clk(c, CLK_Q24);
    mk_sync();
    MRegs<CF> R;
    mk_load_regs<CF>(q, R);
    if (c.stamp && tid == 0) c.stamp[1] = global_ns();
    mk_clk(c, CLK_REGS);
    MShared* sh = c.sh;
    bool first = true;
    for (int u = blockIdx.x; u < S.nunits; u += gridDim.x) {
        for (int j = 0; j < S.per0; j++) {  // gate/up rows 64u + j*RC ..
            const float* rb = mk_chunk<CF>(p, c, nb, RC, R, first);
            first = false;
            if (!rb) return false;
            if (tid < RC / 2) {
                const int r0 = 2 * tid;
                float gv = 0.f, uv = 0.f;
#pragma unroll
                for (int w = 0; w < WPR; w++) {
                    gv += rb[r0 * WPR + w];
                    uv += rb[(r0 + 1) * WPR + w];
                }
                sh->act[(j * RC + r0) / 2] = (p.geglu ? gelu_ref_f(gv) : silu_ref_f(gv)) * uv;
            }
        }
        mk_sync();
        if (warp == 0) {  // the act block as q24 (lanes 0-7: four elements each)
            Q24 aq;
            aq.pl = sh->aq;
            aq.cb = &sh->acb;
            aq.sb = &sh->asb;
            aq.nb = 1;
            const float4 v = lane < 8 ? reinterpret_cast<const float4*>(sh->act)[lane]
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            mk_q24_quad(aq, 0, lane < 8, v, lane);
        }
        mk_sync();
        uint4 xa[3], xb[3];
#pragma unroll
        for (int pl = 0; pl < 3; pl++) {
            xa[pl] = sh->aq[pl * 2 + 0];
            xb[pl] = sh->aq[pl * 2 + 1];
        }
        const int acb = sh->acb;
        const float asb = sh->asb;
        for (int k = 0; k < S.per1; k++) {  // down rows k*MK_DOWN_ROWS ..
            const int r0 = k * MK_DOWN_ROWS, rows = min(MK_DOWN_ROWS, S.N2 - r0);
            const int rs = c.seq % MK_SLOTS;
            const unsigned par = (unsigned)((c.seq / MK_SLOTS) & 1);
            const bool ok = mbar_wait(&sh->full[rs], par, MK_WAIT_NS);  // agreed on below
            const unsigned char* pay = c.ring + (size_t)rs * MK_SLOT_BYTES;
            const __half* scs = reinterpret_cast<const __half*>(pay + (size_t)rows * 16);
            for (int r = tid; r < rows; r += MK_THREADS) {
                const uint4 w4 = reinterpret_cast<const uint4*>(pay)[r];
                const float d = __half2float(scs[r]);
                const float part = fmaf(d * asb, mk_block_dot(w4, xa, xb, acb), 0.f);
                const long long fx = __float2ll_rn(part * MK_FIX);
                if (ok)
                    atomicAdd(reinterpret_cast<unsigned long long*>(acc_at(S.acc_out, r0 + r)),
                              (unsigned long long)fx);
            }
            if (mk_sync_or(!ok)) {  // slot consumed
                mk_fail(p, c);
                return false;
            }
            mk_release(c, 1);
            c.seq++;
        }
    }
    if (c.stamp && tid == 0) c.stamp[2] = global_ns();
    mk_clk(c, CLK_MAIN);
    return true;
}

// ---- attention stage: QK-norm + RoPE + K/V write + split-KV attention -----------
// Pull the cached K/V rows [jlo, min(jhi, pos)) of attention unit u (kv head
// u % n_kv, key split u / n_kv of n_active) of the layer at kc / vc into L2.
__device__ __forceinline__ void mk_kv_prefetch_unit(const MParams& p, const float* kc,
                                                    const float* vc, int u, int n_active,
                                                    int pos, int window) {
    const int g = u % p.n_kv, split = u / p.n_kv;
    int jlo, jhi;
    attn_range(pos + 1, window, split, n_active, &jlo, &jhi);
    const int j1 = min(jhi, pos);
    if (j1 <= jlo) return;
    const float* kb = kc + (size_t)g * p.max_seq * p.hd;
    const float* vb = vc + (size_t)g * p.max_seq * p.hd;
    prefetch_l2(kb + (size_t)jlo * p.hd, kb + (size_t)j1 * p.hd);
    prefetch_l2(vb + (size_t)jlo * p.hd, vb + (size_t)j1 * p.hd);
}

// Thread 0 of a CTA: pull the cached K/V rows of the attention units it will
// run into L2 while the stage before it runs (layer 0; later layers are
// prefetched by the CTAs idle in the previous layer's attention stage, off
// every critical path).
__device__ inline void mk_kv_prefetch(const MParams& p, const MStage& A, const MCtx& c) {
    const int seq = c.pos + 1;
    const int n_active = attn_active_splits(attn_span(seq, A.window), p.n_splits, p.attn_min);
    for (int u = blockIdx.x; u < p.n_kv * n_active; u += gridDim.x)  // every unit of this CTA
        mk_kv_prefetch_unit(p, A.kc, A.vc, u, n_active, c.pos, A.window);
}

template <int EPL, int GMAX>
__device__ inline bool mk_attn(const MParams& p, const MStage& S, MCtx& c) {
    const int G = p.n_heads / p.n_kv, hd = p.hd, half = hd / 2;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int pos = c.pos, seq = pos + 1;
    const int n_active = attn_active_splits(attn_span(seq, S.window), p.n_splits, p.attn_min);
    const int units = p.n_kv * n_active;
    const int qd = p.n_heads * hd, kvd = p.n_kv * hd;
    float* sm = reinterpret_cast<float*>(c.work);
    float* res = sm + (size_t)MK_WARPS * G * (hd + 2);
    float* cwt = sm + (size_t)(MK_WARPS + 1) * G * (hd + 2);
    float* qs = cwt + (size_t)G * (p.n_splits + 1);
    float* ks = qs + (size_t)G * hd;
    if ((int)blockIdx.x >= units) {  // no unit here: prefetch the next layer's K/V rows
        const int f = blockIdx.x - units;
        if (tid == 0 && S.layer + 1 < p.n_layers) {
            // the next layer's window (layers alternate in windowed families)
            const int nw = S.window ? 0 : p.window_next;
            const int na = attn_active_splits(attn_span(seq, nw), p.n_splits, p.attn_min);
            const size_t ls = (size_t)p.n_kv * p.max_seq * hd;  // one layer of the cache
            if (f < p.n_kv * na) mk_kv_prefetch_unit(p, S.kc + ls, S.vc + ls, f, na, pos, nw);
        }
        return true;
    }
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
        const int g = u % p.n_kv, split = u / p.n_kv;
        int jlo, jhi;
        attn_range(seq, S.window, split, n_active, &jlo, &jhi);
        const bool holds = pos >= jlo && pos < jhi;
        const int nrows = G + (holds ? 1 : 0);  // <= 5 rows, one per warp
        // this warp's q/k row (the unit holding this step's position also the
        // k and v rows it appends to the cache) from the QKV stage, with no
        // barrier or counter between: each lane polls its tagged words until
        // they carry this (step, layer)'s tag; the norm gains are requested first
        const int r = warp;
        const bool isq = r < G, has_row = r < nrows;
        const float* nw = isq ? S.q_norm : S.k_norm;
        float vv[EPL], wv[EPL];
#pragma unroll
        for (int e = 0; e < EPL; e++) {
            const int d = lane + 32 * e;
            wv[e] = (has_row && d < hd && nw) ? __ldg(nw + d) : 0.f;
        }
        float vnew = 0.f;
        {
            const unsigned tag = c.tag0 + S.layer;
            const unsigned long long* src =
                isq ? p.qkv + (size_t)(g * G + r) * hd : p.qkv + qd + (size_t)g * hd;
            const unsigned long long* vsrc = p.qkv + qd + kvd + (size_t)g * hd + tid;
            const bool wantv = holds && tid < hd;
            unsigned long long w[EPL], wn = 0;
            uint64_t t0 = 0;
            for (unsigned it = 1;; it++) {
                bool all = true;
#pragma unroll
                for (int e = 0; e < EPL; e++) {
                    const int d = lane + 32 * e;
                    const bool in = has_row && d < hd;
                    w[e] = in ? ld_relaxed_u64(src + d) : 0ull;
                    all = all && (!in || (unsigned)(w[e] >> 32) == tag);
                }
                if (wantv) {
                    wn = ld_relaxed_u64(vsrc);
                    all = all && (unsigned)(wn >> 32) == tag;
                }
                if (all) break;
                if ((it & 15) == 0) {  // bounded as mk_wait_count
                    const uint64_t now = global_ns();
                    if (t0 == 0) t0 = now;
                    if (ld_volatile_i32(p.status) != 0 || now - t0 > MK_WAIT_NS) {
                        atomicExch(p.status, (int)DEV_TIMEOUT);
                        *reinterpret_cast<volatile int*>(&c.sh->abort) = 1;
                        break;
                    }
                }
            }
#pragma unroll
            for (int e = 0; e < EPL; e++) vv[e] = __uint_as_float((unsigned)w[e]);
            vnew = __uint_as_float((unsigned)wn);
        }
        if (has_row) {  // QK-norm (qwen3.rs:154-155)
            float* dst = isq ? qs + (size_t)r * hd : ks;
            if (nw) {
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < EPL; e++) ss = fmaf(vv[e], vv[e], ss);
                ss = warp_sum(ss);
                const float inv = 1.0f / sqrtf(ss / (float)hd + p.eps);
#pragma unroll
                for (int e = 0; e < EPL; e++) vv[e] = __fmul_rn(__fmul_rn(vv[e], inv), wv[e]);
            }
#pragma unroll
            for (int e = 0; e < EPL; e++) {
                const int d = lane + 32 * e;
                if (d < hd) dst[d] = vv[e];
            }
        }
        mk_clk(c, CLK_LOADED);  // attention: inputs arrived, QK-norm done
        mk_sync();
        if (c.sh->abort) return false;
        for (int i = tid; i < nrows * half; i += MK_THREADS) {  // RoPE (rope.wgsl:25-34)
            const int rr = i / half, kq = i - rr * half;
            float* row = rr < G ? qs + (size_t)rr * hd : ks;
            const float sn = c.sh->rsin[kq], cs = c.sh->rcos[kq];
            const float lo = row[kq], hi = row[kq + half];
            row[kq] = __fsub_rn(__fmul_rn(lo, cs), __fmul_rn(hi, sn));
            row[kq + half] = __fadd_rn(__fmul_rn(hi, cs), __fmul_rn(lo, sn));
        }
        mk_sync();
        mk_clk(c, CLK_NORMED);  // attention: RoPE done
        float* kbase = S.kc + (size_t)g * p.max_seq * hd;
        float* vbase = S.vc + (size_t)g * p.max_seq * hd;
        if (holds && tid < hd) {  // cache.rs:21-24
            kbase[(size_t)pos * hd + tid] = ks[tid];
            vbase[(size_t)pos * hd + tid] = vnew;
        }
        mk_sync();
        mk_clk(c, CLK_Q24);  // attention: new K/V row stored
        if (c.stamp && tid == 0) c.stamp[1] = global_ns();
        attn_core<EPL, GMAX, KV_CG, MK_WARPS, true, mk_attn_u(EPL)>(
            qs, G, hd, kbase, vbase, hd, jlo, jhi, p.scale, p.attn_softcap, sm, res);
        mk_clk(c, CLK_REGS);  // attention: this split's state merged
        if (c.stamp && tid == 0) c.stamp[2] = global_ns();
        if (n_active >= 2 && n_active <= MK_DEFER) {
            const int W = hd + 2, WP = mk_part_w(hd);
            for (int i = tid; i < G * W; i += MK_THREADS) {
                const int gi = i / W, d = i - gi * W;
                p.part[((size_t)(g * G + gi) * p.part_stride + split) * WP + d] = res[i];
            }
        } else {
            attn_finish(res, G, hd, g, split, n_active, p.part_stride, p.part, p.counters, p.attn,
                        cwt, MK_THREADS, true);
        }
        mk_sync();
        // this unit's state (or, from the merging unit, the head's output) is
        // stored: release it to the O-projection units of the kv head
        if (tid == 0) red_release_add_u32(p.ardy + (size_t)S.layer * p.n_kv + g, 1u);
        mk_clk(c, CLK_MAIN);  // attention: output (or partial) published
    }
    return true;
}

// ---- O projection by columns: one query head x RC output rows per unit --------------
// Unit (h, rows [r0, r0 + RC)): warp 0 forms head h's attention output
// (mk_head_out4: the split merge) as NBH = head_dim/32 q24 blocks, then the
// CTA dots them with the head's column blocks of W_o for its rows -- one
// row's NBH blocks on NBH consecutive lanes, summed in a fixed order -- and
// adds each row's partial sum into the fixed-point accumulator S.acc_out.
// Every residual row so receives one addition per query head, and a unit
// needs only its own head's attention state, not the whole attention output.
template <int NBH>
__device__ inline bool mk_ocol(const MParams& p, const MStage& S, MCtx& c) {
    static_assert(NBH == 1 || NBH == 2 || NBH == 4 || NBH == 8, "head_dim 32 .. 256");
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nch = (S.N + S.RC - 1) / S.RC;
    const int na = attn_active_splits(attn_span(c.pos + 1, S.window), p.n_splits, p.attn_min);
    bool first = true;
    for (int u = blockIdx.x; u < S.nunits; u += gridDim.x) {
        const int h = u / nch, r0 = (u - h * nch) * S.RC, rows = min(S.RC, S.N - r0);
        const Q24 aq = q24_carve(c.work, NBH);
        if (warp == 0) {  // lane: block lane/8, elements 4*(lane%8) .. +3
            // every attention unit of this head's kv group has published
            if (lane == 0)
                mk_wait_count(p, c, p.ardy + (size_t)S.layer * p.n_kv + h / (p.n_heads / p.n_kv),
                              (unsigned)na);
            __syncwarp();
#pragma unroll
            for (int b0 = 0; b0 < NBH; b0 += 4) {  // four blocks per pass
                const int b = b0 + (lane >> 3);
                const float4 v = b < NBH ? mk_head_out4(p.attn, p.part, p.part_stride, p.hd, h,
                                                        b * 32 + 4 * (lane & 7), na)
                                         : f4_zero();
                mk_q24_quad(aq, b, b < NBH, v, lane);
            }
        }
        if (first) mk_clk(c, CLK_LOADED);
        mk_sync();
        if (c.sh->abort) return false;
        if (first) {
            mk_clk(c, CLK_Q24);
            if (c.stamp && tid == 0) c.stamp[1] = global_ns();
        }
        bool ok = true;
        for (int k = 0; k < S.per0; k++) {
            const int q = c.seq + k;
            ok = mbar_wait(&c.sh->full[q % MK_SLOTS], (unsigned)((q / MK_SLOTS) & 1), MK_WAIT_NS) && ok;
        }
        if (first) mk_clk(c, CLK_WAITED);
        for (int i0 = 0; i0 < S.RC * NBH; i0 += MK_THREADS) {
            const int i = i0 + tid, row = i / NBH, k = i % NBH;
            float part = 0.f;
            if (row < rows) {
                const int sj = k / S.per1, ii = k - sj * S.per1;
                const unsigned char* pay = c.ring + (size_t)((c.seq + sj) % MK_SLOTS) * MK_SLOT_BYTES;
                const size_t e = (size_t)ii * rows + row;  // [block][row], then the scales
                const uint4 w4 = reinterpret_cast<const uint4*>(pay)[e];
                const float d = __half2float(
                    reinterpret_cast<const __half*>(pay + (size_t)S.per1 * rows * 16)[e]);
                uint4 xa[3], xb[3];
#pragma unroll
                for (int pl = 0; pl < 3; pl++) {
                    xa[pl] = aq.pl[(pl * 2 + 0) * NBH + k];
                    xb[pl] = aq.pl[(pl * 2 + 1) * NBH + k];
                }
                part = fmaf(d * aq.sb[k], mk_block_dot(w4, xa, xb, aq.cb[k]), 0.f);
            }
#pragma unroll
            for (int o = 1; o < NBH; o <<= 1) part += __shfl_xor_sync(FULL, part, o);
            if (k == 0 && row < rows && ok)
                atomicAdd(reinterpret_cast<unsigned long long*>(acc_at(S.acc_out, r0 + row)),
                          (unsigned long long)__float2ll_rn(part * MK_FIX));
        }
        if (mk_sync_or(!ok)) {  // slots consumed
            mk_fail(p, c);
            return false;
        }
        mk_release(c, S.per0);
        c.seq += S.per0;
        if (first && c.stamp && tid == 0) c.stamp[2] = global_ns();
        first = false;
    }
    mk_clk(c, CLK_MAIN);
    return true;
}

// GEMV work mapping by config index and slots per chunk.
template <int I, int NS> struct CfgOfT;
template <> struct CfgOfT<0, 1> { using T = MC0; };
template <> struct CfgOfT<1, 1> { using T = MC1; };
template <> struct CfgOfT<2, 1> { using T = MC2; };
template <> struct CfgOfT<3, 1> { using T = MC3; };
template <> struct CfgOfT<4, 1> { using T = MC4; };
template <> struct CfgOfT<0, 2> { using T = MD0; };
template <> struct CfgOfT<1, 2> { using T = MD1; };
template <> struct CfgOfT<2, 2> { using T = MD2; };
template <> struct CfgOfT<3, 2> { using T = MD3; };
template <> struct CfgOfT<4, 2> { using T = MD4; };
template <int I, int NS> using CfgOf = typename CfgOfT<I, NS>::T;

// The step kernel, specialised for one model shape: EPL = head_dim / 32
// registers per lane and GMAX >= n_heads / n_kv for the attention stage (EPL
// column blocks per head in the O projection), CD the GEMV config of K = dim
// (QKV, FFN gate/up, LM head), POST the post-norm residual of Gemma-2-like
// families.  Only the code one model runs is compiled into its kernel, which
// keeps the instruction footprint small.
template <int EPL, int GMAX, int CD, bool POST>
__global__ void __launch_bounds__(MK_BLOCK, 1) k_step(MParams p) {
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ MShared sh;
    __shared__ float rowred[128];
    __shared__ __align__(16) MStage sst[3];  // stage si in sst[si % 3], two fetched ahead
    MCtx c;
    c.sh = &sh;
    c.ring = smem;
    c.work = smem + (size_t)MK_SLOTS * MK_SLOT_BYTES;
    c.emb = reinterpret_cast<float*>(c.work + p.work_bytes);
    MIssue* iss = reinterpret_cast<MIssue*>(c.work + p.work_bytes + al16((size_t)p.dim * 4));
    c.iss = iss;
    c.rowred = rowred;
    c.seq = 0;
    c.redsel = 0;
    c.nch = 0;
    c.stamp = nullptr;
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < MK_SLOTS; s++) {
            mbar_init(&sh.full[s], 1);
            mbar_init(&sh.empty[s], 1);
        }
        fence_mbar_init();
        sh.issued = 0;
        sh.abort = 0;
        sh.prod_done = 0;
        sh.pol = l2_evict_first();
    }
    for (int i = tid; i < p.n_stages * 4; i += MK_BLOCK)
        reinterpret_cast<int4*>(iss)[i] = reinterpret_cast<const int4*>(p.issues)[i];
    __syncthreads();  // every thread, the producer warp included
    if (tid >= MK_THREADS) {  // the producer warp: the step's weight copies, in order
        if (tid == MK_ISSUER) mk_produce(p, c);
        return;
    }
    mk_load_stage(p, 0, &sst[0]);
    mk_load_stage(p, 1, &sst[1]);
    mk_load_stage_wait();
    const int pos = p.st->pos;
    const unsigned tok = p.st->token;
    const unsigned long long base = p.st->bar_base;
    // QKV word tags: (step's first grid-barrier index) + 1 + layer.  The
    // barrier count only grows and a step passes more barriers (two per
    // layer) than it has layers, so no (step, layer) reuses a tag of a word
    // still in the buffer; the session clears the buffer (tag 0) at its start.
    c.tag0 = (unsigned)(base / gridDim.x) + 1u;
    // fault injection (tests of the timeout path): the first grid barrier
    // waits for a count no CTA reaches and gives up after stall_us
    const unsigned stall_us = p.st->stall_us;
    c.pos = pos;
    if (tid < p.hd / 2)  // rope.wgsl:25-34: angle pos * theta^(-2k/hd), f32
        sincosf(__fmul_rn((float)pos, __ldg(p.inv_freq + tid)), &sh.rsin[tid], &sh.rcos[tid]);
    mk_sync();
    // embedding row (qwen3.rs:128-133), every CTA its own copy
    {
        const int nb = p.dim / 32;
        for (int i = tid; i < p.dim; i += MK_THREADS) {
            const int b = i >> 5, j = i & 31;
            const size_t blk = (size_t)tok * nb + b;
            const float d = __half2float(p.emb_scales[blk]);
            const uint8_t byte = p.emb_payload[blk * 16 + (j & 15)];
            const int qv = (j < 16) ? (byte & 0xf) : (byte >> 4);
            float v = __fmul_rn(d, (float)(qv - 8));
            if (p.embed_scale > 0.f) v = __fmul_rn(v, p.embed_scale);
            c.emb[i] = v;
        }
        mk_sync();
    }
    bool ok = true;
    unsigned nbar = 0;  // grid barriers passed this step
    for (int si = 0; si < p.n_stages && ok; si++) {
        if (si > 0) {
            // the attention stage polls the tagged QKV words and the
            // O-projection stage waits on the attention-done counters
            // instead; the CTA barrier publishes the stage descriptor
            const int kind = iss[si].kind;
            if (kind == SK_ATTN || kind == SK_OCOL) {
                mk_sync();
            } else {
                nbar++;
                if (stall_us && nbar == 1)
                    ok = mk_grid_sync(p, c, base + (unsigned long long)(nbar + 1) * gridDim.x,
                                      (uint64_t)stall_us * 1000ull);
                else
                    ok = mk_grid_sync(p, c, base + (unsigned long long)nbar * gridDim.x);
            }
        }
        if (!ok) break;
        unsigned long long* stamp =
            p.stamps ? p.stamps + ((size_t)si * gridDim.x + blockIdx.x) * MK_STAMPS : nullptr;
        c.stamp = stamp;
        if (stamp && tid == 0) stamp[0] = global_ns();
        mk_clk(c, CLK_START);
        mk_load_stage(p, si + 2, &sst[(si + 2) % 3]);  // waited for at the stage end
        const MStage& S = sst[si % 3];
        const MStage& S1 = sst[(si + 1) % 3];
        if (tid == 0 && si + 1 < p.n_stages &&
            S1.kind == SK_ATTN && S1.layer == 0)
            mk_kv_prefetch(p, S1, c);
        mk_clk(c, CLK_AHEAD);
        if (S.kind == SK_ATTN) {
            ok = mk_attn<EPL, GMAX>(p, S, c);
        } else if (S.kind == SK_OCOL) {
            ok = mk_ocol<EPL>(p, S, c);
        } else if (S.kind == SK_FFN) {
            ok = mk_ffn<CfgOf<CD, 2>, POST>(p, S, c);
        } else if (S.epi == EPI_HEAD) {  // always two slots per chunk
            ok = mk_gemv<CfgOf<CD, 2>, EPI_HEAD, POST>(p, S, c);
        } else {
            ok = S.cfg >= MK_NCFG ? mk_gemv<CfgOf<CD, 2>, EPI_STORE, POST>(p, S, c)
                                  : mk_gemv<CfgOf<CD, 1>, EPI_STORE, POST>(p, S, c);
        }
        mk_load_stage_wait();  // made visible by the next stage's CTA barrier
        if (stamp) {
            mk_sync();
            if (tid == 0) stamp[3] = global_ns();
            mk_clk(c, CLK_END);
        }
    }
    mk_load_stage_wait();
    mk_drain(c);
    if (!ok || sh.abort) return;
    // the last CTA to finish clears what the next step expects at zero (the
    // ready counters, the last layer's accumulators) and does the
    // generate-loop bookkeeping (mod.rs:114-122)
    if (tid == 0) {
        __threadfence();
        sh.last = atomicAdd(&p.st->done, 1u) == gridDim.x - 1;
    }
    mk_sync();
    if (sh.last) {
        __threadfence();
        const int nc = p.n_layers * p.n_kv;
        for (int i = tid; i < nc; i += MK_THREADS) p.ardy[i] = 0;
        for (int i = tid; i < p.dim; i += MK_THREADS) {
            *acc_at(p.zero_a, i) = 0;
            *acc_at(p.zero_b, i) = 0;
        }
        mk_sync();
    }
    if (sh.last && tid == 0) {
        {
            __threadfence();
            DevState* st = p.st;
            unsigned next;
            if (pos + 1 < st->n_prompt) {
                next = p.prompt[pos + 1];
            } else {
                const unsigned long long k = atomicMax(&st->key, 0ull);
                const unsigned t = p.decode ? argmax_key_index(k) : 0u;
                p.toks[st->n_produced] = t;
                st->n_produced = st->n_produced + 1;
                next = t;
            }
            st->key = argmax_key_init();
            st->token = next;
            st->pos = pos + 1;
            st->done = 0;
            st->bar_base = base + (unsigned long long)nbar * gridDim.x;
            __threadfence();
        }
    }
}


using StepKernel = void (*)(MParams);

}  // namespace cw
