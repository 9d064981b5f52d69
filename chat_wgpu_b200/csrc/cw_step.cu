// cw_step.cu -- host side of the persistent decode step: the stage plan,
// the kernel variant table, the cooperative launch and the stage profile.
// The device code is in cw_step.cuh; each kernel variant is instantiated in
// its own cw_step_k*.cu so they compile in parallel.
#include <algorithm>
#include <cstdlib>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "cw_step.cuh"

namespace cw {

// ---- host ---------------------------------------------------------------------------
// Column-block-major copy of a packed Q4_0 matrix: block b of row r moves to
// [b][r], so the column block an FFN unit needs is one contiguous range.
__global__ void k_colmajor(const uint8_t* __restrict__ pay, const __half* __restrict__ sc, int rows,
                           int nb, uint8_t* __restrict__ opay, __half* __restrict__ osc) {
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)rows * nb) return;
    const int r = (int)(i / nb), b = (int)(i - (long)r * nb);
    reinterpret_cast<uint4*>(opay)[(size_t)b * rows + r] = reinterpret_cast<const uint4*>(pay)[i];
    osc[(size_t)b * rows + r] = sc[i];
}

static int build_down_colmajor(cw_model* m) {
    if (!m->down_cm.empty()) return CW_OK;
    cw_ctx* ctx = m->ctx;
    std::vector<QW> out;
    for (const Layer& l : m->L) {
        const int rows = l.down.rows, nb = l.down.in_f / 32;
        const size_t pb = (size_t)rows * nb * 16, sb = (size_t)rows * nb * 2;
        const size_t soff = (pb + 255) / 256 * 256;
        cw_buf b;
        BufEntry* e;
        CW_TRY(buf_new(ctx, soff + sb, BUF_PERSISTENT, &b, &e));
        m->owned.push_back(b);
        QW q;
        q.payload = reinterpret_cast<const uint8_t*>(e->ptr);
        q.scales = reinterpret_cast<const __half*>(reinterpret_cast<char*>(e->ptr) + soff);
        q.rows = rows;
        q.in_f = l.down.in_f;
        q.buf = b;
        const long n = (long)rows * nb;
        k_colmajor<<<(unsigned)((n + 255) / 256), 256, 0, ctx->stream>>>(
            l.down.payload, l.down.scales, rows, nb, const_cast<uint8_t*>(q.payload),
            const_cast<__half*>(q.scales));
        CW_CUDA(cudaGetLastError());
        out.push_back(q);
    }
    CW_CUDA(cudaStreamSynchronize(ctx->stream));
    m->down_cm.swap(out);
    return CW_OK;
}
struct StepPlan {
    std::vector<const char*> names;  // stage names, for the profile
    MStage* d_stages = nullptr;
    int n_stages = 0;  // decode step (prompt steps drop the final LM-head stage)
    MParams params{};
    size_t smem = 0;
    int grid = 0;
    void (*kern)(MParams) = nullptr;
};

// Kernel variants (head_dim / 32, GQA group bound, config of K = dim,
// config of K = q-dim): Qwen3-0.6B, Qwen3-1.7B, Qwen3-4B/8B, Llama-3.2-1B-like
// shapes, and the two small test shapes.  Other shapes use the per-stage
// kernels.
#define CW_STEP_VARIANTS(X) \
    X(4, 2, 0, 1) X(4, 2, 1, 1) X(4, 4, 2, 2) X(2, 4, 1, 1) X(2, 2, 0, 0) X(1, 4, 0, 0)
#define CW_STEP_DECL(E, G, D, Q) StepKernel step_kernel_##E##_##G##_##D##_##Q();
CW_STEP_VARIANTS(CW_STEP_DECL)
#undef CW_STEP_DECL

static int gmax_of(int G) { return G <= 1 ? 1 : G <= 2 ? 2 : G <= 4 ? 4 : 8; }

static StepKernel find_kernel(const cw_model_info& I) {
    const int G = I.n_heads / I.n_kv;
    const int epl = (I.head_dim + 31) / 32, gmax = gmax_of(G);
    const int cd = mk_cfg_for(I.dim), cq = mk_cfg_for(I.n_heads * I.head_dim);
#define CW_STEP_FIND(E, G_, D, Q) \
    if (epl == E && gmax == G_ && cd == D && cq == Q) return step_kernel_##E##_##G_##_##D##_##Q();
    CW_STEP_VARIANTS(CW_STEP_FIND)
#undef CW_STEP_FIND
    return nullptr;
}

static size_t work_bytes_for(const cw_model_info& I, int n_splits) {
    const int G = I.n_heads / I.n_kv, hd = I.head_dim;
    const int kmax = std::max<int>(I.dim, std::max<int>(I.n_heads * I.head_dim, I.hidden));
    // PRO_X: q24 planes of K <= kmax; PRO_NORM (K = dim): planes + hbuf + wbuf
    const int qd = I.n_heads * I.head_dim;
    const size_t gemv = std::max({al16(q24_bytes(kmax / 32)),
                                  al16(q24_bytes((int)I.dim / 32)) + (size_t)I.dim * 8,
                                  al16(q24_bytes(qd / 32)) + (size_t)I.n_heads * (MK_DEFER + 1) * 4});
    const size_t attn = (attn_smem_floats(G, hd, n_splits, MK_WARPS) + (size_t)G * hd + hd) * 4;
    return al16(std::max(gemv, attn));
}

bool step_supported(const cw_model* m, const cw_session* s) {
    const cw_model_info& I = m->info;
    if (I.post_norms || I.sliding_window || I.attn_softcap > 0.f || I.final_softcap > 0.f ||
        I.activation != 0 || I.norm_kind != 0)
        return false;
    if (I.head_dim % 32 || I.n_heads % I.n_kv || !find_kernel(I)) return false;
    const int ks[3] = {(int)I.dim, (int)(I.n_heads * I.head_dim), (int)I.hidden};
    for (int K : ks)
        if (K % 256 || mk_cfg_for(K) < 0) return false;
    (void)s;
    return true;
}

int step_plan_create(cw_session* s) {
    cw_model* m = s->m;
    cw_ctx* ctx = s->ctx;
    const cw_model_info& I = m->info;
    if (!step_supported(m, s)) return CW_ERR_UNSUPPORTED;
    std::unique_ptr<StepPlan> P(new StepPlan());
    P->kern = find_kernel(I);
    const int grid = ctx->sm_count;
    const int n_splits = std::max(1, std::min(s->n_splits, grid / (int)I.n_kv));
    CW_TRY(build_down_colmajor(m));
    // ---- stage list and its weight-copy schedule
    std::vector<MStage> st;
    std::vector<MIssue> is;
    auto gemv = [&](const char* name, const QW& w, int pro, int epi, const float* x,
                    const float* base, const float* norm_w, float* y, const float* bias,
                    float* xn_out, int acc_in, int acc_zero) {
        P->names.push_back(name);
        MStage S = {};
        S.acc_in = acc_in;
        S.acc_zero = acc_zero;
        S.racc = s->racc;
        S.kind = SK_GEMV;
        S.cfg = mk_cfg_for(w.in_f);
        // two slots per chunk where a CTA would otherwise take several chunks
        if ((w.rows + mk_rc(S.cfg) - 1) / mk_rc(S.cfg) > grid) S.cfg += MK_NCFG;
        S.pro = pro;
        S.epi = epi;
        S.K = w.in_f;
        S.N = w.rows;
        S.RC = mk_rc(S.cfg);
        S.nchunks = (S.N + S.RC - 1) / S.RC;
        S.payload = w.payload;
        S.scales = w.scales;
        S.x = x;
        S.base = base;
        S.norm_w = norm_w;
        S.y = y;
        S.bias = bias;
        S.xn_out = xn_out;
        st.push_back(S);
        MIssue I = {};
        I.kind = SK_GEMV;
        I.pay0 = S.payload;
        I.sc0 = S.scales;
        I.n0 = S.nchunks;
        I.rc = S.RC / mk_ns(S.cfg);
        I.per0 = mk_ns(S.cfg);
        I.nb = S.K / 32;
        I.n = S.N;
        is.push_back(I);
    };
    for (uint32_t li = 0; li < I.n_layers; li++) {
        const Layer& l = m->L[li];
        gemv("attn_in", l.qkv, PRO_NORM, EPI_STORE, nullptr, li == 0 ? nullptr : s->hidden,
             l.attn_norm, s->qkv, l.qkv_bias, nullptr, li > 0, 0);
        P->names.push_back("attention");
        MStage A = {};
        A.kind = SK_ATTN;
        A.q_norm = l.q_norm;
        A.k_norm = l.k_norm;
        A.kc = s->kc + (size_t)li * I.n_kv * s->max_seq * I.head_dim;
        A.vc = s->vc + (size_t)li * I.n_kv * s->max_seq * I.head_dim;
        st.push_back(A);
        MIssue IA = {};
        IA.kind = SK_ATTN;
        is.push_back(IA);
        // the residual read here includes the previous layer's FFN output
        // (fixed-point accumulator), which is folded in and cleared
        gemv("attn_out", l.wo, PRO_ATTN, EPI_RESID, s->attn, nullptr, nullptr, s->hidden, nullptr,
             nullptr, li > 0, 1);
        P->names.push_back("ffn");
        const QW& dcm = m->down_cm[li];
        MStage F = {};
        F.kind = SK_FFN;
        F.cfg = mk_cfg_for(l.gate_up.in_f) + MK_NCFG;
        F.pro = PRO_NORM;
        F.K = l.gate_up.in_f;
        F.N = l.gate_up.rows;
        F.RC = mk_rc(F.cfg);
        F.nunits = (int)I.hidden / 32;
        F.per0 = 64 / F.RC;
        F.per1 = ((int)I.dim + MK_DOWN_ROWS - 1) / MK_DOWN_ROWS;
        F.N2 = (int)I.dim;
        F.racc = s->racc;
        F.payload = l.gate_up.payload;
        F.scales = l.gate_up.scales;
        F.payload2 = dcm.payload;
        F.scales2 = dcm.scales;
        F.base = s->hidden;
        F.norm_w = l.ffn_norm;
        st.push_back(F);
        MIssue IF = {};
        IF.kind = SK_FFN;
        IF.pay0 = F.payload;
        IF.sc0 = F.scales;
        IF.pay1 = F.payload2;
        IF.sc1 = F.scales2;
        IF.n0 = F.nunits;
        IF.rc = F.RC / mk_ns(F.cfg);
        IF.nb = F.K / 32;
        IF.n = F.N;
        IF.per0 = 64 / IF.rc;
        IF.per1 = F.per1;
        IF.dim = F.N2;
        is.push_back(IF);
    }
    gemv("lm_head", m->head, PRO_NORM, EPI_HEAD, nullptr, s->hidden, m->final_norm, s->logits,
         nullptr, s->xnorm, I.n_layers > 0, 0);
    P->n_stages = (int)st.size();
    // ---- shared memory: ring | work | embedding row | issue table
    const size_t work = work_bytes_for(I, n_splits);
    P->smem = (size_t)MK_SLOTS * MK_SLOT_BYTES + work + al16((size_t)I.dim * 4) +
              is.size() * sizeof(MIssue);
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
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, P->kern, MK_THREADS, P->smem);
    if (e != cudaSuccess || per_sm < 1)
        return set_error(CW_ERR_UNSUPPORTED, "persistent step cannot be resident: %s",
                         cudaGetErrorString(e));
    P->grid = grid;
    const size_t sb = st.size() * sizeof(MStage), ib = is.size() * sizeof(MIssue);
    e = cudaMalloc(&P->d_stages, sb + ib);
    if (e == cudaSuccess)
        e = cudaMemcpy(P->d_stages, st.data(), sb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy(reinterpret_cast<char*>(P->d_stages) + sb, is.data(), ib,
                       cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        if (P->d_stages) cudaFree(P->d_stages);
        return set_error(CW_ERR_CUDA, "persistent step plan: %s", cudaGetErrorString(e));
    }
    MParams& pp = P->params;
    pp.stages = P->d_stages;
    pp.issues = reinterpret_cast<const MIssue*>(reinterpret_cast<char*>(P->d_stages) + sb);
    pp.st = s->st;
    pp.status = ctx->d_status;
    pp.bar = s->bar;
    pp.emb_payload = m->embed.payload;
    pp.emb_scales = m->embed.scales;
    pp.embed_scale = I.embed_scale;
    pp.hidden = s->hidden;
    pp.qkv = s->qkv;
    pp.attn = s->attn;
    pp.prompt = s->prompt;
    pp.toks = s->toks;
    pp.part = s->part;
    pp.counters = s->counters;
    pp.inv_freq = m->inv_freq;
    pp.dim = (int)I.dim;
    pp.n_heads = (int)I.n_heads;
    pp.n_kv = (int)I.n_kv;
    pp.hd = (int)I.head_dim;
    pp.max_seq = (int)s->max_seq;
    pp.n_splits = n_splits;
    pp.part_stride = s->n_splits;
    pp.attn_min = MK_ATTN_MIN;
    if (const char* ev = getenv("CW_ATTN_MIN_KEYS")) {  // tuning knob
        const int v = atoi(ev);
        if (v >= 1) pp.attn_min = v;
    }
    pp.eps = I.eps;
    pp.inv_dim = 1.0f / (float)I.dim;
    pp.scale = powf((float)I.head_dim, -0.5f);  // attention.rs:18
    pp.work_bytes = work;
    s->plan = P.release();
    return CW_OK;
}

void step_plan_free(cw_session* s) {
    if (!s->plan) return;
    if (s->plan->d_stages) cudaFree(s->plan->d_stages);
    delete s->plan;
    s->plan = nullptr;
}

static int step_launch(cw_session* s, bool decode, unsigned long long* stamps) {
    StepPlan* P = s->plan;
    MParams pp = P->params;
    pp.stamps = stamps;
    pp.decode = decode ? 1 : 0;
    pp.n_stages = decode ? P->n_stages : P->n_stages - 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)P->grid);
    cfg.blockDim = dim3(MK_THREADS);
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
    const size_t n = (size_t)P->n_stages * P->grid * MK_STAMPS;
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
        unsigned long long prev_end = 0;
        for (int si = 0; si < P->n_stages; si++) {
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
            auto& w = (*agg)[P->names[si]];
            w.first += 1;
            w.second += (double)(t1 - t0) * 1e-6;
            double dmax = 0;  // the slowest CTA's own duration (span minus start skew)
            for (int b = 0; b < P->grid; b++) {
                const unsigned long long* q = &h[((size_t)si * P->grid + b) * MK_STAMPS];
                if (q[1]) dmax = std::max(dmax, (double)(q[3] - q[0]));
            }
            auto& wm = (*agg)[std::string(P->names[si]) + ".cta_max"];
            wm.first += 1;
            wm.second += dmax * 1e-6;
            static const char* phase[3] = {"prologue", "main", "epilogue"};
            for (int k = 0; k < 3 && nw; k++) {
                auto& r = (*agg)[std::string(P->names[si]) + "." + phase[k]];
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
                auto& r = (*agg)[std::string(P->names[si]) + ":" + clk[k]];
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
                auto& r = (*agg)[std::string(P->names[si]) + ":" + ck[k]];
                r.first += 1;
                r.second += c3[k] / n3 / (double)ctx->clock_khz;
            }
            if (si > 0) {
                auto& g = (*agg)["grid_barrier"];
                g.first += 1;
                g.second += (double)(t0 - prev_end) * 1e-6;
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
