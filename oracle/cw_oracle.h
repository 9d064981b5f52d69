/*
 * cw_oracle.h -- CPU restatement of EggerMarc/chat-wgpu's decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker that the CUDA path is
 * compared against.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / --impl reference legs may load it.  The product library
 * (chat_wgpu_b200/libchatcuda.so) never links or calls it.
 *
 * Every function cites the reference file:line whose arithmetic it restates
 * (paths are relative to the chat-wgpu source tree).  Floating point follows
 * the reference's f32 semantics: the library is compiled with
 * -ffp-contract=off so a*b+c is two roundings, as in the reference's Rust CPU
 * code.
 */
#ifndef CW_ORACLE_H
#define CW_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- dequantisation (src/loader/dequant.rs) ---------------------------- */
float orc_f16_to_f32(uint16_t h);                                   /* :9-21   */
float orc_bf16_to_f32(uint16_t h);                                  /* :23-25  */
void orc_dequant_f16(const uint8_t* b, size_t n, float* out);       /* :37-39  */
void orc_dequant_q8_0(const uint8_t* b, size_t n, float* out);      /* :46-58  */
void orc_dequant_q4_0(const uint8_t* b, size_t n, float* out);      /* :62-78  */
void orc_dequant_q4_1(const uint8_t* b, size_t n, float* out);      /* :82-97  */
void orc_dequant_q6_k(const uint8_t* b, size_t n, float* out);      /* :102-131 */
/* Q4_K / Q5_K: not in the reference (dequant.rs:6, ROADMAP.md:52-53); ggml's
 * published block_q4_K / block_q5_K layout restated (cw_oracle.c). */
void orc_dequant_q4_k(const uint8_t* b, size_t n, float* out);
void orc_dequant_q5_k(const uint8_t* b, size_t n, float* out);

/* ---- q4 re-quantiser + GEMVs ------------------------------------------ */
/* src/kernels/q4.rs:37-60 */
void orc_quantize_q4_0(const float* data, size_t out_f, size_t in_f,
                       float* scales, uint32_t* quants);
/* src/main.rs:133-150 (CPU dequant-and-dot of the crate's q4 layout) */
void orc_q4_gemv(const float* x, const float* scales, const uint32_t* quants,
                 size_t in_f, size_t out_f, float* y);
/* GGUF Q4_0 weight [out_f, in_f] applied to x: dequant_q4_0
 * (src/loader/dequant.rs:62-78) then the dense GEMV of
 * src/kernels/matmul.wgsl:43-50 (sequential k order). */
void orc_q4_0_gemv(const float* x, const uint8_t* blocks, size_t in_f,
                   size_t out_f, float* y);
/* examples/bench/src/lib.rs:221-233 */
void orc_matmul(const float* a, const float* b, size_t m, size_t k, size_t n,
                float* c);

/* ---- elementwise / norm / rope / attention / argmax -------------------- */
/* src/kernels/norm.wgsl:20-56; unit != 0 selects rmsnorm_unit (1 + w) */
void orc_rmsnorm(const float* x, const float* w, size_t rows, size_t dim,
                 float eps, int unit, float* y);
/* src/kernels/rope.wgsl:25-34 */
void orc_rope(const float* x, size_t rows, size_t head_dim, uint32_t pos,
              float theta, float* y);
/* src/kernels/attention.wgsl:23-96 with scale from attention.rs:18.
 * q [n_heads*hd], k/v [seq, n_kv*hd] (row stride n_kv*hd). */
void orc_attention(const float* q, const float* k, const float* v,
                   size_t n_heads, size_t n_kv, size_t seq, size_t head_dim,
                   float* out);
/* Same, plus the Gemma-2 behaviours that have no reference code (restated,
 * not reference): tanh soft-capping of the scaled scores (softcap > 0) and a
 * sliding window over the last `window` keys (window > 0). */
void orc_attention_ext(const float* q, const float* k, const float* v,
                       size_t n_heads, size_t n_kv, size_t seq,
                       size_t head_dim, float softcap, uint32_t window,
                       float* out);
void orc_add(const float* a, const float* b, size_t n, float* c); /* ewise.wgsl:9-13 */
void orc_swiglu(const float* g, const float* u, size_t n, float* out); /* glu.wgsl:25,33-36 */
void orc_geglu(const float* g, const float* u, size_t n, float* out);  /* glu.wgsl:27-30,38-42 */
uint32_t orc_argmax(const float* logits, size_t n);               /* argmax.wgsl:18-55 */

/* ---- GGUF + model ------------------------------------------------------- */
typedef struct orc_model orc_model;

/* Parse a GGUF v3 file (src/loader/gguf.rs:68-106) and bind a family:
 * "qwen3" (src/model/qwen3.rs:44-99), "qwen2"/"llama" (same composition
 * without QK-norm), "gemma2" (restated, not reference).  Returns NULL and
 * fills err on failure. */
orc_model* orc_model_open(const char* path, char* err, size_t errlen);
void orc_model_close(orc_model* m);
/* Model dimensions: dim, n_layers, n_heads, n_kv, head_dim, hidden, vocab. */
void orc_model_dims(const orc_model* m, uint32_t* out7);

/* Greedy generation with the semantics of src/model/mod.rs:57-125: the prompt
 * runs one token per step, the argmax at the last prompt position is the first
 * produced token, exactly max_new tokens are produced.  If logits_out is not
 * NULL it receives the logits of every step that produced a token,
 * [max_new, vocab].  Returns 0 on success. */
int orc_generate(orc_model* m, const uint32_t* prompt, size_t n_prompt,
                 size_t max_new, uint32_t* out_tokens, float* logits_out);

/* One forward step of the model at `pos` for `token`, with the KV state kept
 * inside the model (src/model/qwen3.rs:139-191).  Call orc_model_reset before
 * a new sequence.  Writes the hidden state after the final norm (dim floats)
 * and, if logits != NULL, the logits (vocab floats). */
int orc_model_reset(orc_model* m, size_t max_seq);
int orc_model_step(orc_model* m, uint32_t token, size_t pos, float* hidden,
                   float* logits);

/* Hook::tap (src/model/mod.rs:155-165): record, at every step, the values the
 * reference's forward hands its hook for layer `layer` -- "q" after QK-norm
 * and RoPE (qwen3.rs:165), "post_attn" (:180), "layer_out" (:188); -1 = off.
 * orc_model_get_tap copies the last step's three vectors. */
int orc_model_set_tap(orc_model* m, long layer);
int orc_model_get_tap(const orc_model* m, float* q, float* post_attn, float* layer_out);

/* OpenMP threads the oracle may use (0 = library default). */
void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
