// cw_model.h -- model and session state shared by the decode paths
// (cw_model.cu: per-stage kernels; cw_step.cu: the persistent step kernel).
#pragma once

#include <cuda_fp16.h>

#include <map>
#include <string>
#include <vector>

#include "cw_common.h"

namespace cw {

// Per-session device state of the generate loop (src/model/mod.rs:57-125):
// everything a step needs to know lives here, so one captured launch
// replays for every token.
struct DevState {
    int pos;                 // position of the next step
    unsigned token;          // input token of the next step
    int n_prompt;
    int n_produced;
    unsigned long long key;  // argmax accumulator of the current step
    unsigned long long bar_base;  // grid-barrier count at the start of the step
    unsigned done;           // CTAs that finished the current step
    unsigned stall_us;       // fault injection (cw_session_inject_stall): 0 = off
    unsigned long long ctr_base;  // persistent step's head counter at the start of the step
    unsigned stopped;             // an EOS token ended the sequence (cw_sample.cu)
    unsigned ar_seq;   // tensor-parallel peer all-reduces completed (cw_tp_p2p.cu)
    unsigned key_seq;  // tensor-parallel argmax-key exchanges completed
    unsigned pad3;
};

struct QW {  // packed Q4_0 weight (type 2), or raw GGUF Q6_K blocks (type 14)
    const uint8_t* payload = nullptr;  // Q4_0: nibble plane; Q6_K: the raw blocks
    const __half* scales = nullptr;    // Q4_0 only
    int rows = 0, in_f = 0;
    cw_buf buf = 0;
    int type = 2;
    // Q6_K / Q8_0: the aligned split the streaming decode GEMV reads (payload
    // plane [rows][in_f/256][208] or [rows][in_f/32][32], and an f16 d
    // plane), beside the raw blocks that the
    // embedding lookups and the other kernels read; null where the streaming
    // GEMV does not take in_f
    const uint8_t* split = nullptr;
    const __half* split_d = nullptr;
};

struct Layer {
    float *attn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *ffn_norm = nullptr;
    float *post_attn = nullptr, *post_ffw = nullptr, *qkv_bias = nullptr;
    QW qkv, wo, gate_up, down;
    // q, k and v of different k-quant types (Q4_K_M files keep some v in Q6_K)
    // stay two or three weights (consecutive ones of one type stacked), each
    // writing its slice of the qkv vector; unused slots have 0 rows
    bool qkv_split = false;
    QW q, k, v;
};



struct StepPlan;  // cw_step.cu

// Hook taps (src/model/mod.rs:155-165, qwen3.rs:165,180,188): a named
// intermediate of one layer copied every step into a device ring of `cap`
// positions (slot pos % cap).
enum TapKind : int { TAP_Q = 0, TAP_POST_ATTN = 1, TAP_LAYER_OUT = 2 };
struct Tap {
    int kind = TAP_Q;
    uint32_t layer = 0;
    size_t cap = 0, len = 0;
    float* ring = nullptr;
    cw_buf buf = 0;
};

}  // namespace cw

struct cw_model {
    cw_ctx* ctx = nullptr;
    cw_model_info info{};
    std::vector<cw::Layer> L;
    float* final_norm = nullptr;
    cw::QW embed, head;
    // persistent step (cw_step.cu): slot-packed copies of the matrices it
    // streams, one contiguous [payload | scales] range per weight-ring slot;
    // built on the first plan, for that plan's slot geometry (pk_key)
    std::vector<const uint8_t*> pk_qkv, pk_gu, pk_down, pk_wo;
    const uint8_t* pk_head = nullptr;
    long long pk_key = -1;
    std::vector<cw_buf> owned;
    const float* inv_freq = nullptr;
    // every projection and the head (4 per layer: qkv, wo, gate_up, down; then
    // the head) in the tensor-core GEMM's packed Q4_0 tile records
    // (cw_gemm.cu), built on first use by prefill or a session group
    std::vector<void*> packed;
    // the same matrices in the streaming group step's tile-interleaved form
    // (cw_mgemv.cu, mg_tile_pack; null where K is beyond its integer-MMA
    // path), built by the first group that streams
    std::vector<void*> grp_tiles;
    // tensor parallelism (cw_model_load_gguf_tp): this rank's share of heads,
    // FFN columns and vocabulary; residual-branch sums all-reduced over NCCL
    int tp_rank = 0, tp_world = 1;
    void* nccl = nullptr;
    cw_model_info info_full{};  // the whole model's shapes (info holds this rank's share)
    uint32_t vocab_full = 0;    // token ids range over the full vocabulary
    uint32_t vocab_offset = 0;  // first vocabulary row of this rank's LM-head shard
};

struct cw_session {
    cw_model* m = nullptr;
    cw_ctx* ctx = nullptr;
    size_t max_seq = 0;
    std::vector<cw_buf> owned;
    float *kc = nullptr, *vc = nullptr;
    float *hidden = nullptr, *hidden_b = nullptr, *tmp = nullptr, *qkv = nullptr, *attn = nullptr;
    float *act = nullptr, *logits = nullptr, *xnorm = nullptr, *part = nullptr;
    unsigned *prompt = nullptr, *toks = nullptr, *counters = nullptr;
    // fixed-point residual accumulators of the persistent step, 4 x dim words:
    // the O-projection and FFN partial sums by layer parity (Y0, Y1, Z0, Z1)
    long long* racc = nullptr;
    float* hid2 = nullptr;    // the persistent step's residual base, two buffers [2][dim]
    unsigned* rdy = nullptr;  // its attention-done counters ([n_layers][n_kv], after a spare half)
    cw::DevState* st = nullptr;
    int n_splits = 1;
    bool use_graph = true;
    // captured steps, [step variant][decode] (one variant in use)
    cudaGraphExec_t graphs[2][2] = {{nullptr, nullptr}, {nullptr, nullptr}};
    size_t host_pos = 0, n_prompt = 0, n_produced = 0;
    unsigned* h_tok = nullptr;     // pinned, one token for per-step reads
    unsigned* h_tok_in = nullptr;  // pinned, one token for per-step writes
    // persistent step kernel (cw_step.cu); null when the model is not eligible
    cw::StepPlan* plan = nullptr;
    bool use_persistent = true;
    unsigned long long* bar = nullptr;  // [0] grid-barrier counter, [1] head counter (monotonic)
    void* pf_mem = nullptr;             // batched-prefill scratch (cw_prefill.cu), grown on demand
    size_t pf_bytes = 0;
    size_t pf_chunk = 0;                // rows per prefill chunk (0 = PF_CHUNK)
    // sampling and stop tokens (cw_sample.cu); temperature 0 = greedy
    float smp_temperature = 0.f, smp_top_p = 1.f;
    unsigned smp_top_k = 0;
    unsigned long long smp_seed = 0;
    std::vector<unsigned> eos;
    void* smp_dev = nullptr;  // SampleParams on the device
    bool stopped = false;     // host view of DevState::stopped
    std::vector<cw::Tap> taps;  // active hook taps (force the per-stage step kernels)
    float* qtap = nullptr;      // the step's normed, rotated q (source of "q" taps)
    // the persistent step's QKV rows as tagged 8-byte words (float | tag << 32)
    unsigned long long* qkv_words = nullptr;
    // tensor parallelism over NVLink peer memory (cw_tp_p2p.cu): the all-
    // reduces of the per-stage step once cw_session_tp_attach mapped every
    // rank's exchange area (cw::TpP2P; null: NCCL)
    void* p2p = nullptr;
};

namespace cw {

// cw_step.cu: persistent one-launch-per-step decode.
bool step_supported(const cw_model* m, const cw_session* s);
// Whether a new session starts on the persistent step: where it is supported
// and measured faster than the per-stage kernels (not for the post-norm
// family: Gemma-2-2B runs 1.49 ms/token on it against 1.29 per-stage, its
// 72-block rows leaving 44 % of the step's GEMV lanes idle).
bool step_default(const cw_model* m, const cw_session* s);
int step_plan_create(cw_session* s);
void step_plan_free(cw_session* s);
int step_enqueue(cw_session* s, bool decode);
int step_variant(const cw_session* s);  // 0 or 1: which plan the next step uses
int step_profile(cw_session* s, size_t n_steps,
                 std::map<std::string, std::pair<uint32_t, double>>* agg);

// cw_prefill.cu: prompt positions [host_pos, n_prompt - 1) in batched chunks
// on the tensor cores; advances host_pos and the device state.
int session_prefill(cw_session* s, size_t* n_done);
// cw_prefill.cu: the packed GEMM copies of the weights (model->packed), idempotent.
int model_pack_weights(cw_model* m);

const Tap* find_tap(const cw_session* s, int kind, uint32_t layer);
int sync_counts(cw_session* s);
// Every projection (and, with `head`, the LM head) is Q4_0: the persistent
// step, batched prefill and session groups take only those.
bool model_q4_only(const cw_model* m, bool head);  // host n_produced / stopped from the device state (syncs)

// cw_sample.cu: device-side sampling / EOS after a decode step's finalize.
int sample_params_size();
int sample_params_write(cw_session* s);  // session settings -> device (syncs)
bool sample_active(const cw_session* s);
int sample_enqueue(cw_session* s);

}  // namespace cw
