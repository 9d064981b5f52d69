// cw_gemv.cu -- host launcher of the streaming Q4 GEMV (cw_gemv.cuh).
#include <algorithm>
#include <cstdlib>
#include <map>
#include <tuple>

#include "cw_gemv.cuh"

namespace cw {

template <int LAYOUT, int PRO, int EPI, class CF>
static int sgemv_go(cw_ctx* ctx, const GemvArgs& a, bool pdl) {
    const int nb = a.K / 32;
    const long nchunks = ((long)a.N + CF::RC - 1) / CF::RC;
    // Small GEMVs (the per-layer decode projections): one chunk per CTA, all
    // weight traffic in flight at once.  Large ones (LM heads): persistent
    // CTAs, as many per SM as registers and shared memory allow, each with a
    // two-stage ring (one chunk landing while the other is consumed).
    auto kern = k_sgemv<LAYOUT, PRO, EPI, CF>;
    // (deeper rings measured slower: they cost CTAs per SM, and the large
    // GEMVs are bound by their consumers, not by bytes in flight)
    const int S = nchunks <= (long)ctx->sm_count * 2 ? 1 : 2;
    const GemvSmem L(CF::RC, CF::WPR, nb, gemv_pbb<LAYOUT>(), gemv_sc_bytes<LAYOUT>(CF::RC, nb), S,
                     a.K, PRO == PRO_NORM);
    CW_CHECK((int)L.total <= ctx->max_smem_optin, CW_ERR_UNSUPPORTED,
             "gemv: K=%d needs %zu bytes of shared memory", a.K, L.total);
    static thread_local std::map<std::tuple<int, const void*, size_t>, int> occ;
    const auto key = std::make_tuple(ctx->device, (const void*)kern, L.total);
    auto it = occ.find(key);
    int per_sm;
    if (it == occ.end()) {
        if (L.total > 48 * 1024)
            CW_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)L.total));
        CW_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, L.total));
        per_sm = std::max(per_sm, 1);
        occ[key] = per_sm;
    } else {
        per_sm = it->second;
    }
    const long grid = std::min<long>(nchunks, (long)ctx->sm_count * per_sm);
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
    if (nb <= GemvC128::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC128>(ctx, a, pdl);
    if (nb <= GemvC192::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC192>(ctx, a, pdl);
    if (nb <= GemvC256::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC256>(ctx, a, pdl);
    if (nb <= GemvC384::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC384>(ctx, a, pdl);
    if constexpr (EPI != EPI_GLU) {  // gate/up pairs need at least two rows per chunk
        if (nb <= GemvC768::NB_MAX) return sgemv_go<LAYOUT, PRO, EPI, GemvC768>(ctx, a, pdl);
    }
    return set_error(CW_ERR_UNSUPPORTED, "gemv: K=%d too large for the streaming kernel", a.K);
}

template <int LAYOUT>
static int sgemv_layout(cw_ctx* ctx, int pro, int epi, const GemvArgs& a, bool pdl) {
    if (pro == PRO_X && epi == EPI_STORE) return sgemv_cfg<LAYOUT, PRO_X, EPI_STORE>(ctx, a, pdl);
    if (pro == PRO_X && epi == EPI_RESID) return sgemv_cfg<LAYOUT, PRO_X, EPI_RESID>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_STORE)
        return sgemv_cfg<LAYOUT, PRO_NORM, EPI_STORE>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_GLU) return sgemv_cfg<LAYOUT, PRO_NORM, EPI_GLU>(ctx, a, pdl);
    if (pro == PRO_NORM && epi == EPI_HEAD)
        return sgemv_cfg<LAYOUT, PRO_NORM, EPI_HEAD>(ctx, a, pdl);
    return set_error(CW_ERR_UNSUPPORTED, "gemv: prologue %d / epilogue %d not instantiated", pro, epi);
}

int launch_sgemv(cw_ctx* ctx, int layout, int pro, int epi, const GemvArgs& a, bool pdl) {
    CW_CHECK(sgemv_supported(layout, a.K), CW_ERR_UNSUPPORTED,
             "gemv: K=%d not handled by the streaming kernel", a.K);
    if (layout == LAYOUT_REF) {
        CW_CHECK(pro == PRO_X && epi == EPI_STORE, CW_ERR_UNSUPPORTED, "gemv: crate layout is x->y only");
        return sgemv_cfg<LAYOUT_REF, PRO_X, EPI_STORE>(ctx, a, pdl);
    }
    if (layout == LAYOUT_Q4K) return sgemv_layout<LAYOUT_Q4K>(ctx, pro, epi, a, pdl);
    if (layout == LAYOUT_Q5K) return sgemv_layout<LAYOUT_Q5K>(ctx, pro, epi, a, pdl);
    if (layout == LAYOUT_Q6K) return sgemv_layout<LAYOUT_Q6K>(ctx, pro, epi, a, pdl);
    if (layout == LAYOUT_Q8) return sgemv_layout<LAYOUT_Q8>(ctx, pro, epi, a, pdl);
    return sgemv_layout<LAYOUT_GGUF>(ctx, pro, epi, a, pdl);
}

}  // namespace cw
