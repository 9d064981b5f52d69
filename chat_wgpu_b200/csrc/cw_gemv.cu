// cw_gemv.cu -- host launcher of the streaming Q4 GEMV (cw_gemv.cuh).
#include <algorithm>
#include <map>
#include <tuple>

#include "cw_gemv.cuh"

namespace cw {

template <int LAYOUT, int PRO, int EPI, class CF>
static int sgemv_go(cw_ctx* ctx, const GemvArgs& a, bool pdl) {
    constexpr int SW = LAYOUT == LAYOUT_GGUF ? 2 : 4;
    const int nb = a.K / 32;
    const long nchunks = ((long)a.N + CF::RC - 1) / CF::RC;
    // Small GEMVs (the per-layer decode projections): one chunk per CTA, all
    // weight traffic in flight at once.  Large ones (LM heads): two
    // persistent CTAs per SM with a ring of up to 4 stages.
    long grid;
    int S;
    if (nchunks <= 2L * ctx->sm_count) {
        grid = nchunks;
        S = 1;
    } else {
        grid = 2L * ctx->sm_count;
        S = (int)std::min<long>(4, (nchunks + grid - 1) / grid);
    }
    GemvSmem L(CF::RC, CF::WPR, nb, SW, S, a.K, PRO == PRO_NORM);
    while (S > 1 && 2 * (L.total + 1024) > (size_t)ctx->smem_per_sm) {
        S--;
        L = GemvSmem(CF::RC, CF::WPR, nb, SW, S, a.K, PRO == PRO_NORM);
    }
    CW_CHECK((int)L.total <= ctx->max_smem_optin, CW_ERR_UNSUPPORTED,
             "gemv: K=%d needs %zu bytes of shared memory", a.K, L.total);
    auto kern = k_sgemv<LAYOUT, PRO, EPI, CF>;
    static thread_local std::map<std::pair<int, const void*>, size_t> attr_set;
    auto key = std::make_pair(ctx->device, (const void*)kern);
    if (L.total > 48 * 1024 && attr_set[key] < L.total) {
        CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)L.total));
        attr_set[key] = L.total;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = ctx->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    GemvArgs args = a;
    if (!args.status) args.status = ctx->d_status;
    CW_CUDA(cudaLaunchKernelEx(&cfg, kern, args, S));
    return CW_OK;
}

template <int LAYOUT, int PRO, int EPI>
static int sgemv_cfg(cw_ctx* ctx, const GemvArgs& a, bool pdl) {
    const int nb = a.K / 32;
    if (nb <= GemvC32::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC32>(ctx, a, pdl);
    if (nb <= GemvC64::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC64>(ctx, a, pdl);
    if (nb <= GemvC96::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC96>(ctx, a, pdl);
    if (nb <= GemvC192::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC192>(ctx, a, pdl);
    if (nb <= GemvC384::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC384>(ctx, a, pdl);
    if constexpr (EPI != EPI_GLU) {  // gate/up pairs need at least two rows per chunk
        if (nb <= GemvC768::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC768>(ctx, a, pdl);
    }
    return set_error(CW_ERR_UNSUPPORTED, "gemv: K=%d too large for the streaming kernel", a.K);
}

int launch_sgemv(cw_ctx* ctx, int layout, int pro, int epi, const GemvArgs& a, bool pdl) {
    CW_CHECK(sgemv_supported(layout, a.K), CW_ERR_UNSUPPORTED,
             "gemv: K=%d not handled by the streaming kernel", a.K);
    if (layout == LAYOUT_REF) {
        CW_CHECK(pro == PRO_X && epi == EPI_STORE, CW_ERR_UNSUPPORTED, "gemv: crate layout is x->y only");
        return sgemv_cfg<LAYOUT_REF, PRO_X, EPI_STORE>(ctx, a, pdl);
    }
    if (pro == PRO_X && epi == EPI_STORE) return sgemv_cfg<LAYOUT_GGUF, PRO_X, EPI_STORE>(ctx, a, pdl);
    if (pro == PRO_X && epi == EPI_RESID) return sgemv_cfg<LAYOUT_GGUF, PRO_X, EPI_RESID>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_STORE)
        return sgemv_cfg<LAYOUT_GGUF, PRO_NORM, EPI_STORE>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_GLU) return sgemv_cfg<LAYOUT_GGUF, PRO_NORM, EPI_GLU>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_HEAD)
        return sgemv_cfg<LAYOUT_GGUF, PRO_NORM, EPI_HEAD>(ctx, a, pdl);
    return set_error(CW_ERR_UNSUPPORTED, "gemv: prologue %d / epilogue %d not instantiated", pro, epi);
}

}  // namespace cw
