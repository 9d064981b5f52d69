/*
 * chatcuda.h -- C ABI of libchatcuda.so, the B200 (sm_100a) replacement for
 * chat-wgpu's GPU layer.
 *
 * The reference reaches the GPU through a Rust `GpuContext` (src/context.rs)
 * and one host wrapper per op (src/kernels/{op}.rs); the model layer
 * (src/model/{mod,qwen3,layers,cache}.rs) only ever calls those.  This header exports the same
 * surface as plain C: an opaque context, buffer handles, one entry point per
 * op wrapper, and the model-level calls.  Each declaration names the
 * reference interface it replaces (path:line in the chat-wgpu tree).
 *
 * Conventions
 *  - Every call returns a cw_status (0 == CW_OK).  On failure a message is
 *    available from cw_last_error() on the calling thread.  Nothing aborts,
 *    traps or throws across the ABI.
 *  - Lengths named `len`/`n` count f32 (or u32) ELEMENTS, as in the reference
 *    (GpuContext::empty(len), copy offsets in f32 elements, context.rs:207,252).
 *    Lengths named `nbytes` count bytes.
 *  - A context is bound to one CUDA device and one stream and, like the
 *    reference's GpuContext (RefCell/Cell, !Sync), must be used from one
 *    thread at a time.
 *  - Ops are enqueued asynchronously on the context's stream, the analogue of
 *    the reference recording into its shared encoder (context.rs:30-33).
 *    cw_read()/cw_read_u32() synchronise, like GpuContext::read.
 *  - Op wrappers return their result in a fresh ARENA buffer (*out), valid
 *    until the next cw_reset_frame()/cw_clear_cache(), exactly as the
 *    reference's ctx.empty() arena slots (context.rs:207-227).
 */
#ifndef CHATCUDA_H
#define CHATCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CW_ABI_VERSION 1

typedef struct cw_ctx cw_ctx;
typedef struct cw_model cw_model;
typedef struct cw_session cw_session;
/* Buffer handle; 0 is "no buffer".  Replaces wgpu::Buffer. */
typedef uint64_t cw_buf;

typedef enum {
    CW_OK = 0,
    CW_ERR_INVALID_ARG = 1,  /* bad handle, size or shape                  */
    CW_ERR_CUDA = 2,         /* a CUDA runtime call failed                 */
    CW_ERR_OOM = 3,          /* device or host allocation failed           */
    CW_ERR_NOT_FOUND = 4,    /* missing file / tensor / metadata           */
    CW_ERR_UNSUPPORTED = 5,  /* dtype, architecture or shape not handled   */
    CW_ERR_TIMEOUT = 6,      /* a bounded device-side wait gave up         */
    CW_ERR_FORMAT = 7,       /* malformed GGUF                             */
    CW_ERR_NO_DEVICE = 8     /* no CUDA device / wrong architecture        */
} cw_status;

/* ---- errors / version --------------------------------------------------- */
/* Message of the last failing call on this thread ("" if none). */
const char* cw_last_error(void);
int cw_abi_version(void);

/* ---- context: src/context.rs ------------------------------------------- */
/* GpuContext::new (context.rs:60-104).  Picks CUDA device `device`, creates a
 * non-blocking stream.  Fails with CW_ERR_NO_DEVICE if the device is not an
 * sm_100 part. */
int cw_ctx_create(int device, cw_ctx** out);
int cw_ctx_destroy(cw_ctx* ctx);
/* GpuContext.backend (context.rs:28,70): e.g. "CUDA sm_100a (NVIDIA B200)". */
int cw_ctx_backend(cw_ctx* ctx, char* buf, size_t cap);
/* Device index and the cudaStream_t (as void*) the context enqueues on. */
int cw_ctx_device(cw_ctx* ctx, int* device);
int cw_ctx_stream(cw_ctx* ctx, void** stream);
/* Launch the decode kernels with programmatic dependent launch (default 1);
 * takes effect for CUDA graphs built afterwards.  No reference counterpart. */
int cw_ctx_set_pdl(cw_ctx* ctx, int on);

/* ---- buffers ------------------------------------------------------------- */
/* GpuContext::storage (context.rs:177-184): upload f32s to a new buffer. */
int cw_storage(cw_ctx* ctx, const float* data, size_t len, cw_buf* out);
/* GpuContext::storage_u32 (context.rs:187-194). */
int cw_storage_u32(cw_ctx* ctx, const uint32_t* data, size_t len, cw_buf* out);
/* Raw bytes (e.g. GGUF blocks); no reference counterpart beyond storage_u32. */
int cw_storage_bytes(cw_ctx* ctx, const void* data, size_t nbytes, cw_buf* out);
/* GpuContext::empty (context.rs:207-227): arena slot `cursor++`, reused at
 * the same slot index every frame while its size is unchanged.  Contents are
 * undefined.  Valid until the next reset_frame / clear_cache. */
int cw_empty(cw_ctx* ctx, size_t len, cw_buf* out);
/* GpuContext::empty_persistent (context.rs:229-232): never recycled. */
int cw_empty_persistent(cw_ctx* ctx, size_t len, cw_buf* out);
/* Drop a storage / persistent buffer (wgpu frees on Drop).  Arena buffers
 * are owned by the context and are rejected here. */
int cw_buf_release(cw_ctx* ctx, cw_buf buf);
/* Size in bytes and device address of a buffer (interop, tests). */
int cw_buf_nbytes(cw_ctx* ctx, cw_buf buf, size_t* nbytes);
int cw_buf_device_ptr(cw_ctx* ctx, cw_buf buf, void** dptr);
/* GpuContext::copy (context.rs:252-269): len f32s from src[src_off..] to
 * dst[dst_off..]; offsets in f32 elements. */
int cw_copy(cw_ctx* ctx, cw_buf src, size_t src_off, cw_buf dst, size_t dst_off, size_t len);
/* queue.write_buffer equivalent: host f32s into dst[dst_off..]. */
int cw_write(cw_ctx* ctx, cw_buf dst, size_t dst_off, const float* data, size_t len);
/* GpuContext::read (context.rs:359-389): flush, wait for the stream, copy
 * len f32s back.  cw_read_u32 is the `.to_bits()` reading of mod.rs:103. */
int cw_read(cw_ctx* ctx, cw_buf src, float* out, size_t len);
int cw_read_u32(cw_ctx* ctx, cw_buf src, uint32_t* out, size_t len);
/* GpuContext::flush (context.rs:139-151): ops are already enqueued, so this
 * only checks for launch errors; it does not wait. */
int cw_flush(cw_ctx* ctx);
/* Wait for all enqueued work; reports device-side errors (CW_ERR_TIMEOUT). */
int cw_sync(cw_ctx* ctx);
/* GpuContext::reset_frame (context.rs:234-240) / clear_cache (:242-250). */
int cw_reset_frame(cw_ctx* ctx);
int cw_clear_cache(cw_ctx* ctx);

/* ---- profiler: src/context.rs:106-126, src/profile.rs ------------------- */
typedef struct {
    char kernel[32];    /* op label, as the reference's pass labels        */
    uint32_t passes;    /* launches                                        */
    double total_ms;    /* summed device time (CUDA events)                */
} cw_profile_row;
/* GpuContext::begin_profile: time every op launched until report. */
int cw_begin_profile(cw_ctx* ctx);
/* GpuContext::report_profile: rows sorted by total descending (profile.rs:114-115). */
int cw_report_profile(cw_ctx* ctx, cw_profile_row* rows, size_t cap, size_t* n_rows);

/* ---- op wrappers: src/kernels/{op}.rs ------------------------------------- */
/* q4::gemv (q4.rs:9-30): y[out_f] = W x with W in the crate's re-quantised
 * layout -- f32 scales[out_f*in_f/32], u32 quants[out_f*in_f/8], sequential
 * nibbles (q4.rs:32-36).  in_f % 32 == 0. */
int cw_q4_gemv(cw_ctx* ctx, cw_buf x, cw_buf scales, cw_buf quants,
               size_t in_f, size_t out_f, cw_buf* out);
/* q4::quantize_q4_0 (q4.rs:37-60) run on the device: f32 w[out_f, in_f] ->
 * new persistent (scales, quants) buffers, bit-identical to the host routine. */
int cw_q4_quantize(cw_ctx* ctx, cw_buf w, size_t out_f, size_t in_f,
                   cw_buf* scales, cw_buf* quants);
/* attention::attention (attention.rs:7-38): single-query GQA attention,
 * q[n_heads*head_dim], k/v [seq, n_kv*head_dim], scale head_dim^-0.5. */
int cw_attention(cw_ctx* ctx, cw_buf q, cw_buf k, cw_buf v, size_t n_heads,
                 size_t n_kv, size_t seq, size_t head_dim, cw_buf* out);
/* The same with the family extensions (no reference code): tanh soft-cap of
 * the scaled scores (softcap > 0) and a sliding window of the last `window`
 * keys (window > 0). */
int cw_attention_ext(cw_ctx* ctx, cw_buf q, cw_buf k, cw_buf v, size_t n_heads,
                     size_t n_kv, size_t seq, size_t head_dim, float softcap,
                     uint32_t window, cw_buf* out);
/* attention::add (attention.rs:40-51): c = a + b. */
int cw_add(cw_ctx* ctx, cw_buf a, cw_buf b, size_t n, cw_buf* out);
/* norm::rmsnorm / norm::rmsnorm_unit (norm.rs:185-195). */
int cw_rmsnorm(cw_ctx* ctx, cw_buf x, cw_buf w, size_t rows, size_t dim, float eps, cw_buf* out);
int cw_rmsnorm_unit(cw_ctx* ctx, cw_buf x, cw_buf w, size_t rows, size_t dim, float eps, cw_buf* out);
/* rope::rope (rope.rs:8-27): rotate-half at position pos. */
int cw_rope(cw_ctx* ctx, cw_buf x, size_t rows, size_t head_dim, size_t pos, float theta, cw_buf* out);
/* activation::swiglu / activation::geglu (activation.rs:42-48). */
int cw_swiglu(cw_ctx* ctx, cw_buf gate, cw_buf up, size_t n, cw_buf* out);
int cw_geglu(cw_ctx* ctx, cw_buf gate, cw_buf up, size_t n, cw_buf* out);
/* argmax::argmax (argmax.rs:11-18): 1-element u32 buffer, ties -> lowest. */
int cw_argmax(cw_ctx* ctx, cw_buf logits, size_t n, cw_buf* out);
/* One sampling draw over logits[n] with the rules of cw_session_set_sampling
 * (draw = the draw index i): 1-element u32 buffer. */
int cw_sample(cw_ctx* ctx, cw_buf logits, size_t n, float temperature, uint32_t top_k,
              float top_p, uint64_t seed, uint64_t draw, cw_buf* out);

/* ---- attention without allocation ----------------------------------------
 * No counterpart in the reference.  For callers that cannot allocate device
 * memory -- a host whose own pool owns every device allocation, or a plugin
 * whose process allocator must not see new blocks: the single-query GQA
 * attention of cw_attention, with q
 * [n_heads*head_dim], k/v [seq, n_kv*head_dim] and out [n_heads*head_dim]
 * passed as device pointers, and the split scratch (partial results and merge
 * counters) kept in one static device array of CW_NOALLOC_SCRATCH_BYTES per
 * GPU that loads the library (held until the process exits).  It calls no
 * cudaMalloc, cudaFree or other allocating routine.  The first call on a
 * device looks up the array's device address (cudaGetSymbolAddress) with that
 * device current; make that first call before any stream capture.  The
 * address is kept for the life of the process: do not call this on a device
 * after a cudaDeviceReset of it.  The calling thread's current device is the
 * same after the call as before it.  Every call
 * shares the array and it keeps the last call's contents: each call clears
 * the counters it uses before its kernel, and calls whose kernels can overlap
 * on the GPU (e.g. on unordered streams) race.  Shapes whose partials exceed
 * the array are rejected with CW_ERR_INVALID_ARG.  The work is enqueued on
 * `stream` (a cudaStream_t; NULL = the legacy default stream); synchronise it
 * before reading `out`.  Results equal cw_attention's for the same inputs. */
#define CW_NOALLOC_SCRATCH_BYTES (1 << 20)
int cw_attention_noalloc(int device, void* stream, const float* q, const float* k,
                         const float* v, float* out, size_t n_heads, size_t n_kv, size_t seq,
                         size_t head_dim);

/* ---- GGUF-native Q4_0 (the B200 weight format) --------------------------
 * GGUF Q4_0 blocks (f16 d + 16 nibble bytes, dequant.rs:60-78) are kept in
 * HBM as two planes: the 16-byte nibble payloads and the f16 scales.  The
 * repack is a lossless byte shuffle, so dequantised weights are bit-exact. */
/* Upload host GGUF Q4_0 blocks of a [rows, in_f] tensor to a new persistent
 * packed weight.  Replaces Q4Linear::from_f32 (layers.rs:82-90) without the
 * lossy re-quantisation. */
int cw_q4_0_upload(cw_ctx* ctx, const void* gguf_blocks, size_t rows, size_t in_f, cw_buf* w);
/* Same from GGUF blocks already on the device (cw_storage_bytes). */
int cw_q4_0_pack(cw_ctx* ctx, cw_buf gguf_blocks, size_t rows, size_t in_f, cw_buf* w);
/* y[out_f] = W x over a packed Q4_0 weight (the decode GEMV). */
int cw_q4_0_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, size_t in_f, size_t out_f, cw_buf* out);
/* Y[rows, out_f] = X[rows, in_f] W^T over a packed Q4_0 weight: the prefill
 * GEMM on the tcgen05 tensor cores (TMA-staged tiles, TMEM accumulators).
 * No counterpart in the reference, whose prompt runs one token at a time
 * through q4::gemv (q4.rs:9-30, mod.rs:78-83); each output row equals that
 * GEMV of the same x row within 1e-3 relative (f16 hi/lo operand split,
 * three MMAs per K step, f32 accumulation).  X f32 row-major; the result is
 * an arena buffer of rows*out_f f32.  rows <= 256 stream the Q4_0 blocks
 * (dequantised in shared memory, split-K partials); larger rows stream W's
 * f16 pair (split once per call).  Uses a context-owned scratch of at most
 * 4*(rows + out_f)*in_f bytes + 32 MB (grown on demand, which synchronises). */
int cw_q4_0_gemm(cw_ctx* ctx, cw_buf x, cw_buf w, size_t rows, size_t in_f, size_t out_f,
                 cw_buf* out);
/* Exact f32 dequantisation of a packed weight (dequant.rs:62-78). */
int cw_q4_0_dequant(cw_ctx* ctx, cw_buf w, size_t rows, size_t in_f, cw_buf* out);
/* The microbenchmark of examples/q4bench.rs for the packed GEMV: `iters`
 * back-to-back launches cycling through the n_w distinct weights ws[] (all
 * [out_f, in_f]; pass enough copies that a weight is evicted from L2 before
 * it comes round again), timed with CUDA events on the context stream.
 * *us_per_launch = device time / iters. */
int cw_q4_0_gemv_bench(cw_ctx* ctx, cw_buf x, const cw_buf* ws, size_t n_w, size_t in_f,
                       size_t out_f, size_t iters, double* us_per_launch);

/* ---- raw GGUF weights: k-quants and the other loader types ---------------
 * The weight is the raw GGUF rows ([rows][in_f/256] groups of 256 weights:
 * one Q4_K / Q5_K / Q6_K super-block of 144 / 176 / 210 bytes, 8 Q8_0 /
 * Q4_1 blocks of 34 / 20 bytes, or 256 F32 / F16 / BF16 values) uploaded
 * with cw_storage_bytes.  Dequantisation is exact to the reference's
 * dequant_q6_k / dequant_q8_0 / dequant_q4_1 / f16_to_f32
 * (dequant.rs:102-131, 46-58, 82-97, 9-21: the types its tensor_f32 takes,
 * gguf.rs:109-121); Q4_K / Q5_K (not implemented by the reference:
 * dequant.rs:6, ROADMAP.md:52-53) follow ggml's published block layout;
 * BF16 is the top half of an f32 (dequant_bf16, dequant.rs:41-43, which the
 * reference's tensor_f32 does not dispatch).  in_f must be a
 * multiple of 256 (at most 16384 for the GEMV). */
#define CW_GGUF_F32 0
#define CW_GGUF_F16 1
#define CW_GGUF_Q4_1 3
#define CW_GGUF_Q8_0 8
#define CW_GGUF_Q4_K 12
#define CW_GGUF_Q5_K 13
#define CW_GGUF_Q6_K 14
#define CW_GGUF_BF16 30
/* y[out_f] = W x (f32 accumulation). */
int cw_kquant_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, int type, size_t in_f, size_t out_f,
                   cw_buf* out);
/* Exact f32 dequantisation of the [rows, in_f] weight. */
int cw_kquant_dequant(cw_ctx* ctx, cw_buf w, int type, size_t rows, size_t in_f, cw_buf* out);
/* The Q6_K weight of dequant_q6_k (dequant.rs:102-131) as the streaming
 * GEMV reads it: the file's 210-byte super-blocks are only 2-byte aligned,
 * so they are split into a [rows][in_f/256][208] plane (ql, qh and the int8
 * scales, as in the file) and a plane of the f16 d values; same bytes in
 * total.  *out is a new persistent buffer (release it with cw_buf_release). */
int cw_q6_k_split(cw_ctx* ctx, cw_buf w, size_t rows, size_t in_f, cw_buf* out);
/* y[out_f] = W x over a cw_q6_k_split weight (in_f a multiple of 256, at most
 * 24576): the sum of w x with w = d * scale * (q - 32) of dequant_q6_k, in
 * integer dot products against the block-floating-point x of the Q4 GEMVs
 * (within 1e-3 relative of the f32 dequantised product). */
int cw_q6_k_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, size_t in_f, size_t out_f, cw_buf* out);
/* The same for Q8_0 (dequant_q8_0, dequant.rs:46-58: w = d * q): its 34-byte
 * blocks split into a [rows][in_f/32][32] plane of int8 codes and a plane of
 * the f16 d values (cw_q8_0_split, a new persistent buffer), and the
 * streaming GEMV over it (in_f a multiple of 256, at most 24576; within 1e-3
 * relative of the f32 dequantised product). */
int cw_q8_0_split(cw_ctx* ctx, cw_buf w, size_t rows, size_t in_f, cw_buf* out);
int cw_q8_0_gemv(cw_ctx* ctx, cw_buf x, cw_buf w, size_t in_f, size_t out_f, cw_buf* out);

/* ---- model: src/model/{mod,qwen3,layers,cache}.rs --------------------------------------------- */
typedef struct {
    uint32_t dim, n_layers, n_heads, n_kv, head_dim, hidden, vocab;
    float eps, rope_theta;
    /* FamilySpec (described by the reference's docs, not implemented there):
     * norm 0 Plain / 1 UnitShift; act 0 SwiGlu / 1 GeGlu. */
    uint32_t norm_kind, activation, qk_norm, qkv_bias, post_norms;
    uint32_t sliding_window;            /* 0 = none; applies to even layers */
    float attn_softcap, final_softcap;  /* 0 = off                          */
    float embed_scale;                  /* 0 = none                         */
    uint64_t weight_bytes;              /* bytes of packed weights in HBM   */
    char arch[16];
} cw_model_info;

/* Model::load (mod.rs:26, qwen3.rs:44-99) from a GGUF file: architectures
 * qwen3 / qwen2 / llama / gemma2; Q4_0 projections and embeddings, F32/F16
 * norms and biases.  Weights stay in their GGUF format in HBM (no
 * re-quantisation).  Projections and untied LM heads may also be Q4_K /
 * Q5_K / Q6_K (the mixes of Q4_K_M-style files, q/k/v of different types
 * included; no reference counterpart, ROADMAP.md:52-53) and token embeddings
 * Q4_K / Q5_K / Q6_K; k-quant projections decode through the per-stage
 * kernels, and
 * cw_session_prefill / cw_group_create / the persistent step take Q4_0
 * projections only. */
int cw_model_load_gguf(cw_ctx* ctx, const char* path, cw_model** out);
/* GgufFile::open (gguf.rs:65-106) without a device: parse the header, the
 * metadata and the tensor table, and check that every tensor's dimensions are
 * non-zero, its byte size does not overflow and it lies inside the file.
 * *n_tensors and *data_bytes (the size of the data section; either may be
 * NULL) describe the file.  CW_ERR_FORMAT for a malformed file (where the
 * reference panics, gguf.rs:192,203,206), CW_ERR_NOT_FOUND when it cannot be
 * opened.  cw_model_load_gguf runs the same checks first. */
int cw_gguf_inspect(const char* path, size_t* n_tensors, uint64_t* data_bytes);
int cw_model_free(cw_model* model);
/* The whole model's shapes (for a tensor-parallel rank too; weight_bytes is
 * what this rank holds). */
int cw_model_get_info(cw_model* model, cw_model_info* info);

/* Tensor-parallel decode (no reference counterpart: the reference runs one
 * model on one adapter).  `world` processes, one GPU each, load the same GGUF
 * with cw_model_load_gguf_tp: rank r keeps heads [r, r+1) * n_heads/world
 * with their KV heads, FFN columns [r, r+1) * hidden/world and LM-head rows
 * [r, r+1) * vocab/world; the O and down partial sums and the argmax are
 * all-reduced over NCCL (libnccl.so.2, opened at run time) inside each step.
 * Every rank drives its session through the same calls in the same order.
 * Greedy decode only: no sampling at temperature > 0, taps, cw_session_prefill
 * or groups; cw_session_logits returns this rank's vocabulary slice.
 * Rank 0 makes the id with cw_tp_unique_id and hands it to the others. */
#define CW_TP_ID_BYTES 128
int cw_tp_unique_id(uint8_t* id, size_t n);
int cw_model_load_gguf_tp(cw_ctx* ctx, const char* path, int rank, int world, const uint8_t* id,
                          cw_model** out);
int cw_model_tp_info(cw_model* model, int* rank, int* world, uint32_t* vocab_offset,
                     uint32_t* vocab_local);
/* The per-stage step's all-reduces over NVLink peer memory instead of NCCL
 * (the O and down partial sums, the argmax key).  Every rank of a session
 * calls cw_session_tp_handle (its exchange area's CUDA IPC handle and its GPU,
 * CW_TP_HANDLE_BYTES), the host hands all of them, in rank order, to every
 * rank's cw_session_tp_attach, which maps the peers' areas.  From then on each
 * all-reduce is one kernel: every element of the partial goes to every peer
 * as one 8-byte NVLink store carrying value and exchange epoch together, each
 * rank waits (bounded: CW_ERR_TIMEOUT after 2 s) for the words of the current
 * epoch and sums them in rank order, identically on every rank.  Ranks must be
 * on distinct GPUs (CW_ERR_UNSUPPORTED otherwise); every rank attaches before
 * its next step and frees its session only after every rank has finished
 * its last step (the host synchronises the ranks). */
#define CW_TP_MAX_WORLD 8
#define CW_TP_HANDLE_BYTES 128
int cw_session_tp_handle(cw_session* s, uint8_t* out, size_t n);
int cw_session_tp_attach(cw_session* s, const uint8_t* handles, size_t n);

/* A decode session = Model::new_cache (qwen3.rs:115) + the per-token state of
 * generate (mod.rs:57-125).  max_seq bounds prompt + generated tokens. */
int cw_session_create(cw_model* model, size_t max_seq, cw_session** out);
int cw_session_free(cw_session* s);
/* Start a sequence: upload the prompt and rewind to position 0. */
int cw_session_begin(cw_session* s, const uint32_t* prompt, size_t n_prompt);
/* Run `n_steps` steps of the generate loop (embed -> forward -> lm_head ->
 * argmax -> next input) on the device without host round trips.  Prompt
 * positions skip the lm_head, whose logits the reference discards
 * (mod.rs:78-81).  Returns the number of tokens produced by these steps. */
int cw_session_run(cw_session* s, size_t n_steps, size_t* n_produced);
/* Batched prefill: run prompt positions [pos, n_prompt - 1) together, the
 * projections as tcgen05 tensor-core GEMMs over the Q4_0 weights (chunks of
 * up to 4096 rows), filling the KV cache exactly where the token-by-token
 * steps would (within 1e-3 relative).  The last prompt token is left for the
 * next cw_session_run/step, which produces the first token as before.  No
 * counterpart in the reference (its prompt runs through forward() one token
 * at a time, mod.rs:78-83).  Allocates a session scratch on first use.
 * *n_done (may be NULL) = positions processed. */
int cw_session_prefill(cw_session* s, size_t* n_done);
/* Rows per cw_session_prefill chunk: 1..4096 (0 = the default, 4096).  Smaller
 * chunks bound the prefill scratch (about 40 KB per row for Qwen3-0.6B
 * shapes) at the cost of more launches; results do not depend on it. */
int cw_session_set_prefill_chunk(cw_session* s, size_t rows);
/* Copy the K and V cache rows [0, n_pos) of `layer` to the host, each laid
 * out [n_kv][n_pos][head_dim] f32 (cache.rs:7-31 holds the same values). */
int cw_session_read_kv(cw_session* s, uint32_t layer, size_t n_pos, float* k, float* v);
/* Co-batched decode (no reference counterpart: its sessions run one at a
 * time).  A group steps n sessions of one model together: one batched step
 * runs every session's next position (prompt or decode, each at its own
 * position with its own KV cache, sampling settings and stop tokens) with
 * each projection and the LM head read once per step for all n rows.  Per
 * session the result equals its own cw_session_run step within 1e-3
 * relative.  Groups of up to 8 sessions of a pre-norm family whose
 * projection widths are multiples of 256 run every projection as one
 * streaming GEMV over all rows (the Q4_0 weights as loaded); other groups
 * run them as tensor-core GEMMs over packed tile records (+0.5625 bytes per
 * weight, built once per model by the first such group).  Sessions must
 * have begun (cw_session_begin) and stay owned by the caller; hook taps are
 * not recorded by group steps.  cw_group_run advances every session by
 * n_steps positions. */
typedef struct cw_group cw_group;
int cw_group_create(cw_session* const* sessions, size_t n, cw_group** out);
int cw_group_free(cw_group* g);
/* Choose the group's projection path: 1 = streaming GEMVs with their
 * products on the integer tensor cores where K <= 4096 (the default of a
 * qualifying group), 2 = streaming GEMVs with dp4a products only (same
 * integer sums), 0 = tensor-core GEMMs over packed tiles, -1 = no change.
 * CW_ERR_UNSUPPORTED when the group does not qualify for streaming.
 * *streaming (may be NULL) receives the path now in use (0, 1 or 2). */
int cw_group_set_streaming(cw_group* g, int on, int* streaming);
int cw_group_run(cw_group* g, size_t n_steps);
/* cw_group_run timed with CUDA events on the context stream (the first step
 * of a new group is captured as a graph and run before the timed region). */
int cw_group_run_timed(cw_group* g, size_t n_steps, double* ms);
/* Tokens produced so far (<= cap). */
int cw_session_tokens(cw_session* s, uint32_t* out, size_t cap, size_t* n);
/* Logits of the last produced token (vocab floats) and the position count. */
int cw_session_logits(cw_session* s, float* out, size_t vocab);
int cw_session_pos(cw_session* s, size_t* pos);
/* Hidden state after the final norm of the last step (dim floats): the
 * analogue of tapping the forward's output (mod.rs:155-165). */
int cw_session_hidden(cw_session* s, float* out, size_t dim);
/* Per-step path selection: 1 = one CUDA graph per token (default),
 * 0 = direct launches (debug). */
int cw_session_set_graph(cw_session* s, int use_graph);
/* Step kernel selection (no reference counterpart: the reference always
 * dispatches one compute pass per op).  1 = the whole step as ONE persistent
 * cooperative launch (default for the shapes it covers: no post-norms, no
 * sliding window, no soft-caps, RMSNorm, SwiGLU, dim/q-dim/hidden multiples
 * of 256, a compiled kernel variant for the head shape); 2 = the same (the
 * split-attention plan, its only plan); 0 = one kernel per stage.  Returns CW_ERR_UNSUPPORTED when a persistent mode is
 * asked for a family it does not cover.  cw_session_persistent reports
 * whether the persistent step is in use. */
int cw_session_set_persistent(cw_session* s, int on);
/* Fault injection for tests of the timeout path (no reference counterpart:
 * the reference has no device-side waits).  The next persistent step waits
 * at its first grid barrier for a count no CTA reaches, gives up after
 * wait_us microseconds, and every CTA leaves early; the next synchronising
 * call (cw_sync, cw_session_tokens, ...) reports CW_ERR_TIMEOUT.  The GPU
 * context stays usable; the session must be restarted with
 * cw_session_begin.  Only for sessions on the persistent step. */
int cw_session_inject_stall(cw_session* s, uint32_t wait_us);
int cw_session_persistent(cw_session* s, int* on);
/* One step with a host round trip, the shape of the reference's loop body
 * (mod.rs:93-103): the input token is copied from the host (token_in, or
 * CW_TOKEN_DEVICE to keep the device-side feedback), the step runs, and the
 * token it produced (UINT32_MAX for a prompt position) is read back. */
#define CW_TOKEN_DEVICE 0xffffffffu
int cw_session_step(cw_session* s, uint32_t token_in, uint32_t* token_out);
/* Sampling after the LM head (no reference code: its decode is greedy and
 * its `temperature` argument is reserved, wasm.rs:57,63; ROADMAP.md:56-57).
 * temperature <= 0: greedy argmax (the default).  Otherwise a token is drawn
 * on the device from softmax(logits / temperature) restricted to the logits
 * >= the top_k-th largest (top_k 0 = all) and then to the nucleus: the
 * highest-probability tokens whose mass reaches top_p (1 = all).  Draw i of
 * a sequence (i = tokens produced before it) uses the 53-bit uniform
 * splitmix64(seed ^ (i+1) * 0x9E3779B97F4A7C15) >> 11; masses are fixed
 * point (p * 2^40), so a draw is reproducible.  Takes effect from the next
 * step; cw_session_begin does not reset it. */
int cw_session_set_sampling(cw_session* s, float temperature, uint32_t top_k, float top_p,
                            uint64_t seed);
/* Stop tokens (at most CW_MAX_EOS; n = 0 clears): when a decode step
 * produces one, it is not counted or appended and the sequence stops --
 * later steps produce nothing -- as the reference's chat loop breaks on its
 * EOS ids before emitting them (wasm.rs:48-51,99-101).  cw_session_step
 * returns the stop token itself once, then CW_TOKEN_DEVICE.  A new
 * cw_session_begin clears the stop. */
#define CW_MAX_EOS 16
/* Hook::tap (mod.rs:155-165): record the forward pass's named intermediate
 * of `layer` at every position -- "q" (normed, rotated queries, n_heads *
 * head_dim floats, qwen3.rs:165), "post_attn" (hidden after the attention
 * residual, dim floats, :180) or "layer_out" (hidden after the FFN residual,
 * :188) -- into a device ring of the last `cap` positions, with copies that
 * are part of the captured step (no host work per token).  A session with
 * taps runs the per-stage step kernels (the persistent step keeps these
 * values in registers and shared memory); cw_session_prefill records them
 * too.  cw_session_read_tap copies the vector of position `pos` (one of the
 * last `cap` positions run) to the host; len must be the tap's length. */
int cw_session_add_tap(cw_session* s, const char* name, uint32_t layer, size_t cap);
int cw_session_clear_taps(cw_session* s);
int cw_session_read_tap(cw_session* s, const char* name, uint32_t layer, size_t pos, float* out,
                        size_t len);
int cw_session_set_eos(cw_session* s, const uint32_t* ids, size_t n);
int cw_session_stopped(cw_session* s, int* stopped);
/* cw_session_run timed with CUDA events on the context stream: *ms is the
 * device time of the n_steps steps. */
int cw_session_run_timed(cw_session* s, size_t n_steps, double* ms);
/* Kernel launches one step makes (prompt and decode steps). */
int cw_session_launches(cw_session* s, size_t* prompt_step, size_t* decode_step);
/* Per-kernel device time of n_steps decode steps: the step is captured once
 * as a CUDA graph with a CUDA-event pair around every kernel (kernels run
 * back to back without overlap in this graph) and replayed n_steps times;
 * rows aggregate by kernel stage name (the reference's WGPU_PROFILE
 * breakdown, mod.rs:74-88, profile.rs:86-117). */
int cw_session_profile(cw_session* s, size_t n_steps, cw_profile_row* rows, size_t cap,
                       size_t* n_rows);

/* model::generate (mod.rs:57-125): greedy, the prompt one token per step,
 * exactly max_new tokens (and one token when max_new == 0, as the reference's
 * post-push check does).  out_tokens holds max(max_new, 1) entries.  Like the
 * reference (ctx.read per token, mod.rs:103) each produced token is read
 * back to the host before the next step is launched. */
int cw_generate(cw_model* model, const uint32_t* prompt, size_t n_prompt,
                size_t max_new, uint32_t* out_tokens);

#ifdef __cplusplus
}
#endif
#endif /* CHATCUDA_H */
