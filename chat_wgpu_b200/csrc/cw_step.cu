// cw_step.cu -- host side of the persistent decode step: the stage plan,
// the kernel variant table, the cooperative launch and the stage profile.
// The device code is in cw_step.cuh; each kernel variant is instantiated in
// its own cw_step_k*.cu so they compile in parallel.
#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "cw_step.cuh"

namespace cw {

// ---- host ---------------------------------------------------------------------------
// Slot-packed copies of the matrices the step streams (layouts in MIssue,
// cw_step.cuh): one contiguous [payload | scales] range per weight-ring slot,
// so the producer lane fills a slot with one bulk copy.  Source: the
// GGUF-split Q4_0 planes (payload [rows][nb][16], scales [rows][nb]).
// Row slabs of RS rows: slab s at byte s*RS*nb*18.
__global__ void k_pack_rows(const uint8_t* __restrict__ pay, const __half* __restrict__ sc, int rows,
                            int nb, int RS, uint8_t* __restrict__ out) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;  // (row, block)
    if (i >= (long)rows * nb) return;
    const int r = (int)(i / nb), b = (int)(i - (long)r * nb);
    const int s = r / RS, ri = r - s * RS, srows = min(RS, rows - s * RS);
    uint8_t* base = out + (size_t)s * RS * nb * 18;
    reinterpret_cast<uint4*>(base)[(size_t)ri * nb + b] = reinterpret_cast<const uint4*>(pay)[i];
    reinterpret_cast<__half*>(base + (size_t)srows * nb * 16)[(size_t)ri * nb + b] = sc[i];
}
// Column groups of G blocks over CH-row slabs: group g, slab c at byte
// (g*rows + c*CH)*G*18, payload [block][row] then scales [block][row].
__global__ void k_pack_cols(const uint8_t* __restrict__ pay, const __half* __restrict__ sc, int rows,
                            int nb, int G, int CH, uint8_t* __restrict__ out) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;  // (row, column block)
    if (i >= (long)rows * nb) return;
    const int r = (int)(i / nb), cb = (int)(i - (long)r * nb);
    const int g = cb / G, k = cb - g * G;
    const int c = r / CH, ri = r - c * CH, crows = min(CH, rows - c * CH);
    uint8_t* base = out + ((size_t)g * rows + (size_t)c * CH) * G * 18;
    reinterpret_cast<uint4*>(base)[(size_t)k * crows + ri] = reinterpret_cast<const uint4*>(pay)[i];
    reinterpret_cast<__half*>(base + (size_t)G * crows * 16)[(size_t)k * crows + ri] = sc[i];
}

// One packed copy of w (rows x in_f Q4_0), owned by the model.  cols: column
// groups of G blocks over CH-row slabs, else row slabs of RS rows.
static int pack_copy(cw_model* m, const QW& w, bool cols, int RS, int G, int CH,
                     const uint8_t** out) {
    cw_ctx* ctx = m->ctx;
    const int nb = w.in_f / 32;
    cw_buf b;
    BufEntry* e;
    CW_TRY(buf_new(ctx, (size_t)w.rows * nb * 18, BUF_PERSISTENT, &b, &e));
    m->owned.push_back(b);
    uint8_t* dst = reinterpret_cast<uint8_t*>(e->ptr);
    const long n = (long)w.rows * nb;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (cols)
        k_pack_cols<<<blocks, 256, 0, ctx->stream>>>(w.payload, w.scales, w.rows, nb, G, CH, dst);
    else
        k_pack_rows<<<blocks, 256, 0, ctx->stream>>>(w.payload, w.scales, w.rows, nb, RS, dst);
    CW_CUDA(cudaGetLastError());
    *out = dst;
    return CW_OK;
}

// The step's packed matrices for one slot geometry: rows per copy of the QKV
// stage (rs_qkv), the LM head (rs_head) and the FFN gate/up (rs_gu); the O
// projection's column blocks per slot (ocpb) and rows per unit (orc).  Built
// once per model; a plan with another geometry rebuilds them (the previous
// copies stay owned by the model).
static int build_packed(cw_model* m, int rs_qkv, int rs_head, int rs_gu, int ocpb, int orc) {
    const long long key = (((((long long)rs_qkv * 4096 + rs_head) * 4096 + rs_gu) * 64 + ocpb) * 4096) + orc;
    if (m->pk_key == key) return CW_OK;
    std::vector<const uint8_t*> qkv, gu, down, wo;
    for (const Layer& l : m->L) {
        const uint8_t *a, *b, *c, *d;
        CW_TRY(pack_copy(m, l.qkv, false, rs_qkv, 1, 1, &a));
        CW_TRY(pack_copy(m, l.gate_up, false, rs_gu, 1, 1, &b));
        CW_TRY(pack_copy(m, l.down, true, 1, 1, MK_DOWN_ROWS, &c));
        CW_TRY(pack_copy(m, l.wo, true, 1, ocpb, orc, &d));
        qkv.push_back(a);
        gu.push_back(b);
        down.push_back(c);
        wo.push_back(d);
    }
    const uint8_t* head = nullptr;
    CW_TRY(pack_copy(m, m->head, false, rs_head, 1, 1, &head));
    CW_CUDA(cudaStreamSynchronize(m->ctx->stream));
    m->pk_qkv.swap(qkv);
    m->pk_gu.swap(gu);
    m->pk_down.swap(down);
    m->pk_wo.swap(wo);
    m->pk_head = head;
    m->pk_key = key;
    return CW_OK;
}

// The stage list of the step.
struct StepVariant {
    std::vector<const char*> names;  // stage names, for the profile
    MStage* d_stages = nullptr;      // stage table + issue table, one allocation
    int n_stages = 0;                // decode step (prompt steps drop the LM-head stage)
    MParams params{};
};

struct StepPlan {
    StepVariant v[1];
    size_t smem = 0;
    int grid = 0;
    void (*kern)(MParams) = nullptr;
};

// Kernel variants (head_dim / 32, GQA group bound, GEMV config of K = dim,
// post-norm residual): Qwen3-0.6B, Qwen3-1.7B, Qwen3-4B/8B, Llama-3.2-1B-like
// shapes, Gemma-2-2B/9B, and the small test shapes.  Other shapes use the
// per-stage kernels.
#define CW_STEP_VARIANTS(X)                                                             \
    X(4, 2, 0, 0) X(4, 2, 1, 0) X(4, 4, 2, 0) X(2, 4, 1, 0) X(2, 2, 0, 0) X(1, 4, 0, 0) \
    X(8, 2, 2, 1) X(2, 2, 0, 1)
#define CW_STEP_DECL(E, G, D, P) StepKernel step_kernel_##E##_##G##_##D##_##P();
CW_STEP_VARIANTS(CW_STEP_DECL)
#undef CW_STEP_DECL

static int gmax_of(int G) { return G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; }

static StepKernel find_kernel(const cw_model_info& I) {
    const int G = I.n_heads / I.n_kv;
    const int epl = (I.head_dim + 31) / 32, gmax = gmax_of(G);
    const int cd = mk_cfg_for(I.dim), post = I.post_norms ? 1 : 0;
#define CW_STEP_FIND(E, G_, D, P) \
    if (epl == E && gmax == G_ && cd == D && post == P) return step_kernel_##E##_##G_##_##D##_##P();
    CW_STEP_VARIANTS(CW_STEP_FIND)
#undef CW_STEP_FIND
    return nullptr;
}



static size_t work_bytes_for(const cw_model_info& I, int n_splits) {
    const int G = I.n_heads / I.n_kv, hd = I.head_dim;
    const int kmax = std::max<int>(I.dim, std::max<int>(I.n_heads * I.head_dim, I.hidden));
    const int qd = I.n_heads * I.head_dim;
    // PRO_X: q24 planes of K <= kmax; PRO_NORM (K = dim): planes + hbuf + wbuf;
    // O-projection stage: one head's q24 blocks
    const size_t gemv = std::max({al16(q24_bytes(kmax / 32)),
                                  al16(q24_bytes((int)I.dim / 32)) + (size_t)I.dim * 8,
                                  al16(q24_bytes(qd / 32))});
    const size_t attn = (attn_smem_floats(G, hd, n_splits, MK_WARPS) + (size_t)G * hd + hd) * 4;
    return al16(std::max(gemv, attn));
}

bool step_default(const cw_model* m, const cw_session* s) {
    return step_supported(m, s) && !m->info.post_norms;
}

bool step_supported(const cw_model* m, const cw_session* s) {
    const cw_model_info& I = m->info;
    // the two families the step composes: pre-norm SwiGLU (Qwen/Llama), and
    // Gemma-2's post-norm GeGLU with (1 + w) gains and alternating windows
    const bool post = I.post_norms != 0;
    if (post ? (I.norm_kind != 1 || I.activation != 1)
             : (I.sliding_window || I.attn_softcap > 0.f || I.final_softcap > 0.f ||
                I.activation != 0 || I.norm_kind != 0))
        return false;
    if (post && I.dim > 4096) return false;  // its residual is formed in one register batch
    if (I.head_dim % 32 || I.head_dim > 256 || I.n_heads % I.n_kv || !find_kernel(I)) return false;
    if (m->embed.type != 2 || !model_q4_only(m, true)) return false;  // Q6_K / k-quant weights
    if (m->tp_world > 1) return false;  // the all-reduces run between kernels
    const int ks[3] = {(int)I.dim, (int)(I.n_heads * I.head_dim), (int)I.hidden};
    for (int K : ks)
        if (K % 256 || mk_cfg_for(K) < 0) return false;
    (void)s;
    return true;
}

// Rows per O-projection unit (query head x row chunk): the smallest of 128,
// 256, 512, 1024 that gives at most one unit per CTA.
static int ocol_rows(const cw_model_info& I, int grid) {
    int rc = 128;
    while (rc < MK_DOWN_ROWS && (long)I.n_heads * ((I.dim + rc - 1) / rc) > grid) rc *= 2;
    return rc;
}

// The stage list, uploaded to the device.  Per layer l (p = l % 2, q = 1 - p):
//   attn_in    residual = H[p] + Y[q] + Z[q] (layer 0: the embedding row)
//              -> rmsnorm -> QKV GEMV (+bias) -> qkv words tagged with the
//              (step, layer); each CTA also stores its slice of the residual
//              to H[q], the next base
//   attention  (no grid barrier: each unit polls its group's tagged rows)
//              QK-norm, RoPE, K/V row write, split-KV attention; the units of
//              each kv head are counted (ardy)
//   o_proj     (no grid barrier: each unit waits for its kv head's units)
//              per (query head, row chunk): that head's split merge and its
//              column blocks of W_o, partial sums added into Y[p]
//   ffn        residual = H[q] + Y[p] -> rmsnorm -> gate/up -> SwiGLU -> its
//              column block of W_down, partial sums added into Z[p]; zeroes
//              Y[q] and Z[q] (its slice of rows)
// and the LM head on H[L%2] + Y + Z of the last layer.  Y and Z are fixed-
// point int64 accumulators (s->racc: Y[0], Y[1], Z[0], Z[1]), H two f32
// buffers (s->hid2); the attention-done counters, and the last layer's Y
// and Z, are zeroed by the last CTA of every step.
static int build_variant(cw_session* s, int grid, int n_splits, size_t work, StepVariant* V,
                         size_t* smem_need) {
    cw_model* m = s->m;
    cw_ctx* ctx = s->ctx;
    const cw_model_info& I = m->info;
    const int dim = (int)I.dim, L = (int)I.n_layers;
    long long* Y[2] = {s->racc, s->racc + dim};
    long long* Z[2] = {s->racc + 2 * dim, s->racc + 3 * dim};
    float* H[2] = {s->hid2, s->hid2 + dim};
    std::vector<MStage> st;
    std::vector<MIssue> is;
    // GEMV stage config: two slots per chunk where a CTA would otherwise take
    // several chunks (always for the LM head: one head variant per kernel)
    auto gemv_cfg = [&](const QW& w, int epi) {
        int cfg = mk_cfg_for(w.in_f);
        if ((w.rows + mk_rc(cfg) - 1) / mk_rc(cfg) > grid || epi == EPI_HEAD) cfg += MK_NCFG;
        return cfg;
    };
    const int nbh = (int)I.head_dim / 32;          // column blocks per query head
    const int orc = ocol_rows(I, grid);            // rows per O-projection unit
    const int ocpb = std::min(nbh, MK_DOWN_ROWS / orc);  // column blocks per ring slot
    {
        const int cq = gemv_cfg(m->L[0].qkv, EPI_STORE), ch = gemv_cfg(m->head, EPI_HEAD);
        const int cg = mk_cfg_for(m->L[0].gate_up.in_f) + MK_NCFG;
        CW_TRY(build_packed(m, mk_rc(cq) / mk_ns(cq), mk_rc(ch) / 2, mk_rc(cg) / 2, ocpb, orc));
    }
    auto gemv = [&](const char* name, const QW& w, const uint8_t* pk, int pro, int epi,
                    float* fold_to, int layer,
                    const float* base, const float* norm_w, float* y, const float* bias,
                    float* xn_out, int acc_in, long long* r1, long long* r2, const float* pa,
                    const float* pf) {
        V->names.push_back(name);
        MStage S = {};
        S.acc_in = acc_in;
        S.racc = r1;
        S.racc2 = r2;
        S.post_a = pa;
        S.post_f = pf;
        S.kind = SK_GEMV;
        S.cfg = gemv_cfg(w, epi);
        S.pro = pro;
        S.epi = epi;
        S.K = w.in_f;
        S.N = w.rows;
        S.RC = mk_rc(S.cfg);
        S.nchunks = (S.N + S.RC - 1) / S.RC;
        S.fold_to = fold_to;
        S.layer = layer;
        S.base = base;
        S.norm_w = norm_w;
        S.y = y;
        S.bias = bias;
        S.xn_out = xn_out;
        st.push_back(S);
        MIssue Is = {};
        Is.kind = SK_GEMV;
        Is.pk0 = pk;
        Is.n0 = S.nchunks;
        Is.rc = S.RC / mk_ns(S.cfg);
        Is.per0 = mk_ns(S.cfg);
        Is.nb = S.K / 32;
        Is.n = S.N;
        is.push_back(Is);
    };
    const bool post = I.post_norms != 0;
    // window of layer li: Gemma-2 alternates sliding-window (even) and global layers
    auto window_of = [&](int li) {
        return (I.sliding_window && li % 2 == 0) ? (int)I.sliding_window : 0;
    };
    for (int li = 0; li < L; li++) {
        const Layer& l = m->L[li];
        const Layer* lprev = li > 0 ? &m->L[li - 1] : nullptr;
        const int p = li % 2, q = 1 - p;
        float* kc = s->kc + (size_t)li * I.n_kv * s->max_seq * I.head_dim;
        float* vc = s->vc + (size_t)li * I.n_kv * s->max_seq * I.head_dim;
        gemv("attn_in", l.qkv, m->pk_qkv[li], PRO_NORM, EPI_STORE, H[q], li, li == 0 ? nullptr : H[p],
             l.attn_norm, s->qkv, l.qkv_bias, nullptr, li == 0 ? 0 : 2, Y[q], Z[q],
             post && lprev ? lprev->post_attn : nullptr, post && lprev ? lprev->post_ffw : nullptr);
        V->names.push_back("attention");
        MStage T = {};
        T.kind = SK_ATTN;
        T.nobar = 1;
        T.layer = li;
        T.window = window_of(li);
        T.q_norm = l.q_norm;
        T.k_norm = l.k_norm;
        T.kc = kc;
        T.vc = vc;
        st.push_back(T);
        MIssue It = {};
        It.kind = SK_ATTN;
        is.push_back(It);
        V->names.push_back("o_proj");
        MStage O = {};
        O.kind = SK_OCOL;
        O.nobar = 1;
        O.layer = li;
        O.window = window_of(li);
        O.K = (int)(I.n_heads * I.head_dim);
        O.N = dim;
        O.RC = orc;
        O.nunits = (int)I.n_heads * ((dim + orc - 1) / orc);
        O.per1 = ocpb;
        O.per0 = nbh / ocpb;
        O.acc_out = Y[p];
        st.push_back(O);
        MIssue Io = {};
        Io.kind = SK_OCOL;
        Io.pk1 = m->pk_wo[li];
        Io.n0 = O.nunits;
        Io.rc = orc;
        Io.nb = nbh;
        Io.per0 = O.per0;
        Io.per1 = ocpb;
        Io.dim = dim;
        is.push_back(Io);
        V->names.push_back("ffn");
        MStage F = {};
        F.kind = SK_FFN;
        F.cfg = mk_cfg_for(l.gate_up.in_f) + MK_NCFG;
        F.pro = PRO_NORM;
        F.K = l.gate_up.in_f;
        F.N = l.gate_up.rows;
        F.RC = mk_rc(F.cfg);
        F.nunits = (int)I.hidden / 32;
        F.per0 = 64 / F.RC;
        F.per1 = (dim + MK_DOWN_ROWS - 1) / MK_DOWN_ROWS;
        F.N2 = dim;
        F.layer = li;
        F.acc_in = 1;
        F.racc = Y[p];
        F.post_a = post ? l.post_attn : nullptr;
        F.zero_a = li == 0 ? nullptr : Y[q];
        F.zero_b = li == 0 ? nullptr : Z[q];
        F.base = H[q];
        F.norm_w = l.ffn_norm;
        F.acc_out = Z[p];
        st.push_back(F);
        MIssue If = {};
        If.kind = SK_FFN;
        If.pk0 = m->pk_gu[li];
        If.pk1 = m->pk_down[li];
        If.n0 = F.nunits;
        If.rc = F.RC / mk_ns(F.cfg);
        If.nb = F.K / 32;
        If.n = F.N;
        If.per0 = 64 / If.rc;
        If.per1 = F.per1;
        If.dim = F.N2;
        is.push_back(If);
    }
    const int lp = (L - 1) % 2;
    gemv("lm_head", m->head, m->pk_head, PRO_NORM, EPI_HEAD, nullptr, L, H[L % 2], m->final_norm, s->logits,
         nullptr, s->xnorm, 2, Y[lp], Z[lp], post ? m->L[L - 1].post_attn : nullptr,
         post ? m->L[L - 1].post_ffw : nullptr);
    V->n_stages = (int)st.size();
    *smem_need = (size_t)MK_SLOTS * MK_SLOT_BYTES + work + al16((size_t)dim * 4) +
                 is.size() * sizeof(MIssue);
    const size_t sb = st.size() * sizeof(MStage), ib = is.size() * sizeof(MIssue);
    cudaError_t e = cudaMalloc(&V->d_stages, sb + ib);
    // stream-ordered with the step launches (the context stream does not wait
    // for the legacy default stream) and complete before st / is die
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(V->d_stages, st.data(), sb, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(reinterpret_cast<char*>(V->d_stages) + sb, is.data(), ib,
                            cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess)
        return set_error(CW_ERR_CUDA, "persistent step plan: %s", cudaGetErrorString(e));
    MParams& pp = V->params;
    pp.stages = V->d_stages;
    pp.issues = reinterpret_cast<const MIssue*>(reinterpret_cast<char*>(V->d_stages) + sb);
    pp.st = s->st;
    pp.status = ctx->d_status;
    pp.bar = s->bar;
    pp.emb_payload = m->embed.payload;
    pp.emb_scales = m->embed.scales;
    pp.embed_scale = I.embed_scale;
    pp.hidden = s->hidden;
    pp.qkv = s->qkv_words;
    pp.attn = s->attn;
    pp.prompt = s->prompt;
    pp.toks = s->toks;
    pp.part = s->part;
    pp.counters = s->counters;
    pp.inv_freq = m->inv_freq;
    pp.dim = dim;
    pp.n_heads = (int)I.n_heads;
    pp.n_kv = (int)I.n_kv;
    pp.hd = (int)I.head_dim;
    pp.max_seq = (int)s->max_seq;
    pp.n_splits = n_splits;
    pp.n_layers = L;
    pp.ardy = s->rdy + (size_t)L * I.n_kv;
    pp.zero_a = Y[lp];
    pp.zero_b = Z[lp];
    pp.part_stride = s->n_splits;
    pp.attn_min = mk_attn_min(((int)I.head_dim + 31) / 32);
    pp.window_next = (int)I.sliding_window;
    pp.unit = I.norm_kind == 1;
    pp.geglu = I.activation == 1;
    pp.attn_softcap = I.attn_softcap;
    pp.final_softcap = I.final_softcap;
    pp.eps = I.eps;
    pp.inv_dim = 1.0f / (float)dim;
    pp.scale = powf((float)I.head_dim, -0.5f);  // attention.rs:18
    pp.work_bytes = work;
    return CW_OK;
}

static void plan_release(StepPlan* P) {
    for (StepVariant& V : P->v)
        if (V.d_stages) cudaFree(V.d_stages);
    delete P;
}

int step_plan_create(cw_session* s) {
    cw_model* m = s->m;
    cw_ctx* ctx = s->ctx;
    const cw_model_info& I = m->info;
    if (!step_supported(m, s)) return CW_ERR_UNSUPPORTED;
    std::unique_ptr<StepPlan, void (*)(StepPlan*)> P(new StepPlan(), plan_release);
    P->kern = find_kernel(I);
    const int grid = ctx->sm_count;
    const int n_splits = std::max(1, std::min(s->n_splits, grid / (int)I.n_kv));
    const size_t work = work_bytes_for(I, n_splits);
    CW_TRY(build_variant(s, grid, n_splits, work, &P->v[0], &P->smem));
    cudaFuncAttributes fa{};
    cudaError_t e = cudaFuncGetAttributes(&fa, P->kern);
    if (e == cudaSuccess && (long)(P->smem + fa.sharedSizeBytes) > (long)ctx->max_smem_optin)
        return set_error(CW_ERR_UNSUPPORTED,
                         "persistent step needs %zu + %zu bytes of shared memory (max %d)", P->smem,
                         (size_t)fa.sharedSizeBytes, ctx->max_smem_optin);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(P->kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)P->smem);
    int per_sm = 0;
    if (e == cudaSuccess)
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, P->kern, MK_BLOCK, P->smem);
    if (e != cudaSuccess || per_sm < 1)
        return set_error(CW_ERR_UNSUPPORTED, "persistent step cannot be resident: %s",
                         cudaGetErrorString(e));
    P->grid = grid;
    s->plan = P.release();
    return CW_OK;
}

void step_plan_free(cw_session* s) {
    if (!s->plan) return;
    plan_release(s->plan);
    s->plan = nullptr;
}

int step_variant(const cw_session* s) {
    (void)s;
    return 0;
}

static int step_launch(cw_session* s, bool decode, unsigned long long* stamps) {
    StepPlan* P = s->plan;
    const StepVariant& V = P->v[step_variant(s)];
    MParams pp = V.params;
    pp.stamps = stamps;
    pp.decode = decode ? 1 : 0;
    pp.n_stages = decode ? V.n_stages : V.n_stages - 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)P->grid);
    cfg.blockDim = dim3(MK_BLOCK);
    cfg.dynamicSmemBytes = P->smem;
    cfg.stream = s->ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    std::unique_ptr<OpScope> sc;
    if (s->ctx->profiling) sc.reset(new OpScope(s->ctx, "decode_step"));
    CW_CUDA(cudaLaunchKernelEx(&cfg, P->kern, pp));
    return CW_OK;
}

int step_enqueue(cw_session* s, bool decode) { return step_launch(s, decode, nullptr); }

// Stage breakdown of n_steps decode steps from the in-kernel stamps: per
// stage, the span from its first CTA's start to its last CTA's end ("work",
// under the stage name) and from there to the next stage's first start
// ("grid_barrier"); "decode_step" is the CUDA-event time of the launch.
int step_profile(cw_session* s, size_t n_steps,
                 std::map<std::string, std::pair<uint32_t, double>>* agg) {
    StepPlan* P = s->plan;
    cw_ctx* ctx = s->ctx;
    int max_stages = 0;
    for (const StepVariant& V : P->v) max_stages = std::max(max_stages, V.n_stages);
    const size_t n = (size_t)max_stages * P->grid * MK_STAMPS;
    unsigned long long* d = nullptr;
    CW_CUDA(cudaMalloc(&d, n * 8));
    std::vector<unsigned long long> h(n);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = CW_OK;
    if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess)
        rc = set_error(CW_ERR_CUDA, "profile events");
    for (size_t it = 0; it < n_steps && rc == CW_OK; it++) {
        if (s->host_pos >= s->max_seq) {
            rc = set_error(CW_ERR_INVALID_ARG, "session is full: position %zu", s->host_pos);
            break;
        }
        const int vsel = step_variant(s);  // before the position advances
        cudaMemsetAsync(d, 0, n * 8, ctx->stream);
        cudaEventRecord(e0, ctx->stream);
        rc = step_launch(s, true, d);
        if (rc != CW_OK) break;
        cudaEventRecord(e1, ctx->stream);
        cudaError_t e = cudaMemcpyAsync(h.data(), d, n * 8, cudaMemcpyDeviceToHost, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        if (e != cudaSuccess) {
            rc = set_error(CW_ERR_CUDA, "profile step: %s", cudaGetErrorString(e));
            break;
        }
        rc = check_device_status(ctx);
        if (rc != CW_OK) break;
        s->host_pos++;
        s->n_produced++;
        float ms = 0.f;
        cudaEventElapsedTime(&ms, e0, e1);
        auto& a = (*agg)["decode_step"];
        a.first += 1;
        a.second += ms;
        unsigned long long prev_end = 0, layer_t0 = 0;
        const StepVariant& V = P->v[vsel];
        for (int si = 0; si < V.n_stages; si++) {
            unsigned long long t0 = ~0ull, t1 = 0;
            double ph[3] = {0, 0, 0};
            int nw = 0;
            for (int b = 0; b < P->grid; b++) {
                const unsigned long long* q = &h[((size_t)si * P->grid + b) * MK_STAMPS];
                t0 = std::min(t0, q[0]);
                t1 = std::max(t1, q[3]);
                if (q[1] && q[2]) {  // a CTA with work in this stage: its phases
                    ph[0] += (double)(q[1] - q[0]);
                    ph[1] += (double)(q[2] - q[1]);
                    ph[2] += (double)(q[3] - q[2]);
                    nw++;
                }
            }
            auto& w = (*agg)[V.names[si]];
            w.first += 1;
            w.second += (double)(t1 - t0) * 1e-6;
            double dmax = 0;  // the slowest CTA's own duration (span minus start skew)
            for (int b = 0; b < P->grid; b++) {
                const unsigned long long* q = &h[((size_t)si * P->grid + b) * MK_STAMPS];
                if (q[1]) dmax = std::max(dmax, (double)(q[3] - q[0]));
            }
            auto& wm = (*agg)[std::string(V.names[si]) + ".cta_max"];
            wm.first += 1;
            wm.second += dmax * 1e-6;
            static const char* phase[3] = {"prologue", "main", "epilogue"};
            for (int k = 0; k < 3 && nw; k++) {
                auto& r = (*agg)[std::string(V.names[si]) + "." + phase[k]];
                r.first += 1;
                r.second += ph[k] / nw * 1e-6;
            }
            // GEMV stages: SM-clock intervals between the CLK points
            static const char* clk[CLK_N - 1] = {"ahead", "loaded", "normed", "q24",
                                                 "regs", "main", "end"};
            double cl[CLK_N - 1] = {0};
            int nc = 0;
            for (int b = 0; b < P->grid; b++) {
                const unsigned long long* q = &h[((size_t)si * P->grid + b) * MK_STAMPS + 4];
                if (!q[CLK_REGS] || !q[CLK_START]) continue;
                for (int k = 0; k < CLK_N - 1; k++) cl[k] += (double)(q[k + 1] - q[k]);
                nc++;
            }
            for (int k = 0; k < CLK_N - 1 && nc; k++) {
                auto& r = (*agg)[std::string(V.names[si]) + ":" + clk[k]];
                r.first += 1;
                r.second += cl[k] / nc / (double)ctx->clock_khz;  // cycles -> ms
            }
            // first chunk: regs -> waited -> summed -> issued
            static const char* ck[3] = {"1st_wait", "1st_math", "1st_issue"};
            double c3[3] = {0, 0, 0};
            int n3 = 0;
            for (int b = 0; b < P->grid; b++) {
                const unsigned long long* q = &h[((size_t)si * P->grid + b) * MK_STAMPS + 4];
                if (!q[CLK_REGS] || !q[CLK_ISSUED]) continue;
                c3[0] += (double)(q[CLK_WAITED] - q[CLK_REGS]);
                c3[1] += (double)(q[CLK_SUMMED] - q[CLK_WAITED]);
                c3[2] += (double)(q[CLK_ISSUED] - q[CLK_SUMMED]);
                n3++;
            }
            for (int k = 0; k < 3 && n3; k++) {
                auto& r = (*agg)[std::string(V.names[si]) + ":" + ck[k]];
                r.first += 1;
                r.second += c3[k] / n3 / (double)ctx->clock_khz;
            }
            // stages opened by a grid barrier: the gap since the previous
            // stage's end (the attention and O-projection stages overlap the
            // stage before them and have none)
            if (si > 0 && t0 >= prev_end) {
                auto& g = (*agg)["grid_barrier"];
                g.first += 1;
                g.second += (double)(t0 - prev_end) * 1e-6;
                auto& gs = (*agg)[std::string("barrier>") + V.names[si]];  // by the stage it opens
                gs.first += 1;
                gs.second += (double)(t0 - prev_end) * 1e-6;
            }
            // the layer's timeline: each stage's first start and last end
            // from the first start of the layer's QKV stage
            if (!strcmp(V.names[si], "attn_in") || !strcmp(V.names[si], "lm_head")) layer_t0 = t0;
            for (int k = 0; k < 2; k++) {
                auto& r = (*agg)[std::string(V.names[si]) + (k ? "@end" : "@start")];
                r.first += 1;
                r.second += (double)((k ? t1 : t0) - layer_t0) * 1e-6;
            }
            prev_end = t1;
        }
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    cudaFree(d);
    return rc;
}

}  // namespace cw
