// Kernel instantiations of ONE block format: this file is compiled once per format with
// -DQMV_FMT_ID=<GGML type id> (the build does so for every format of formats.py), so the formats build in
// parallel and a change to one kernel family does not rebuild the others.
#include "qmv_host.cuh"
#include "qmv_moe.cuh"

#ifndef QMV_FMT_ID
#error "compile with -DQMV_FMT_ID=<GGML type id>"
#endif

namespace qmv {
namespace {

template <int FMT, int T, bool SUMS>
int launch_t(const MvParams& P, cudaStream_t st) {
    constexpr int RW = 2;
    constexpr int R = SUMS ? 1 : RW;
    const long long groups = (long long)((P.n_out + R - 1) / R) * P.slots;
    long long blocks = (groups + kWarpsPerBlock - 1) / kWarpsPerBlock;
    const long long cap = (long long)sm_count() * 16;
    if (blocks > cap) blocks = cap;
    mv_kernel<FMT, T, R, SUMS><<<unsigned(blocks), 32 * kWarpsPerBlock, 0, st>>>(P);
    return launched();
}

template <int FMT>
int launch_fmt(const MvParams& P, int T, cudaStream_t st) {
    switch (T) {
    case 1: return launch_t<FMT, 1, false>(P, st);
    case 2: return launch_t<FMT, 2, false>(P, st);
    case 3: return launch_t<FMT, 3, false>(P, st);
    case 4: return launch_t<FMT, 4, false>(P, st);
    case 5: return launch_t<FMT, 5, false>(P, st);
    case 6: return launch_t<FMT, 6, false>(P, st);
    case 7: return launch_t<FMT, 7, false>(P, st);
    case 8: return launch_t<FMT, 8, false>(P, st);
    }
    return ST_BAD_TOKENS;
}


template <int FMT, int NCW, int G, int UPL, int XF, bool SUMS>
int launch_tma_k(const TmaParams& P, int grid, int smem, cudaStream_t st) {
    auto kern = mv_tma_kernel<FMT, NCW, G, UPL, XF, SUMS>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess)
            return launched();
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(32 * (NCW + 1));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = (pdl_enabled() && !SUMS) ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kern, P) != cudaSuccess) return launched();
    return launched();
}

template <int FMT, int NCW, int XF, bool SUMS>
int launch_tma_g(const TmaParams& P, const TmaPlan& pl, int grid, cudaStream_t st) {
    switch (pl.G) {
    case 16: return launch_tma_k<FMT, NCW, 16, 1, XF, SUMS>(P, grid, pl.smem, st);
    case 32: return launch_tma_k<FMT, NCW, 32, 1, XF, SUMS>(P, grid, pl.smem, st);
    case 64: return launch_tma_k<FMT, NCW, 64, 1, XF, SUMS>(P, grid, pl.smem, st);
    case 128: return launch_tma_k<FMT, NCW, 128, 1, XF, SUMS>(P, grid, pl.smem, st);
    case 256:
        return pl.UPL == 1 ? launch_tma_k<FMT, NCW, 256, 1, XF, SUMS>(P, grid, pl.smem, st)
                           : launch_tma_k<FMT, NCW, 256, 2, XF, SUMS>(P, grid, pl.smem, st);
    case 512:
        if constexpr (NCW >= 16)
            return pl.UPL == 1 ? launch_tma_k<FMT, NCW, 512, 1, XF, SUMS>(P, grid, pl.smem, st)
                               : launch_tma_k<FMT, NCW, 512, 2, XF, SUMS>(P, grid, pl.smem, st);
    }
    return ST_BAD_SHAPE;
}

template <int FMT, int XF, bool SUMS>
int launch_tma_x(const TmaParams& P, const TmaPlan& pl, int grid, cudaStream_t st) {
#ifdef QMV_SWEEP
    if (pl.NCW == 8) return launch_tma_g<FMT, 8, XF, SUMS>(P, pl, grid, st);
#endif
    return pl.NCW == 16 ? launch_tma_g<FMT, 16, XF, SUMS>(P, pl, grid, st) : ST_BAD_SHAPE;
}

}  // namespace

template <int FMT>
int launch_mv_fmt(const MvParams& P, int T, cudaStream_t st) {
    switch (T) {
    case 1: return launch_t<FMT, 1, false>(P, st);
    case 2: return launch_t<FMT, 2, false>(P, st);
    case 3: return launch_t<FMT, 3, false>(P, st);
    case 4: return launch_t<FMT, 4, false>(P, st);
    case 5: return launch_t<FMT, 5, false>(P, st);
    case 6: return launch_t<FMT, 6, false>(P, st);
    case 7: return launch_t<FMT, 7, false>(P, st);
    case 8: return launch_t<FMT, 8, false>(P, st);
    }
    return ST_BAD_TOKENS;
}

template <int FMT>
int launch_sums_fmt(const MvParams& P, cudaStream_t st) {
    return launch_t<FMT, 1, true>(P, st);
}

template <int FMT>
int launch_tma_fmt(int xf, bool sums, const TmaParams& P, const TmaPlan& pl, int grid, cudaStream_t st) {
    if constexpr (!staged_format(FMT)) return ST_BAD_FORMAT;        // the warp-per-row kernel takes these
    if (sums) return xf == 0 ? launch_tma_x<FMT, 0, true>(P, pl, grid, st) : ST_BAD_SHAPE;
    switch (xf) {
    case 0: return launch_tma_x<FMT, 0, false>(P, pl, grid, st);
    case 1: return launch_tma_x<FMT, 1, false>(P, pl, grid, st);
    case 2: return launch_tma_x<FMT, 2, false>(P, pl, grid, st);
    }
    return ST_BAD_SHAPE;
}

// grid: the work items (an upper bound); launched as min(items, resident CTAs), each CTA looping
template <int FMT>
int launch_moe_fmt(int stage, const MoeParams& P, int grid, cudaStream_t st) {
    static int occ[2] = {0, 0};
    auto kern = stage == 0 ? moe_gateup_kernel<FMT> : moe_down_kernel<FMT>;
    if (occ[stage] == 0) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kMoeThreads, 0) != cudaSuccess || n < 1) n = 1;
        occ[stage] = n;
    }
    grid = std::max(1, std::min(grid, occ[stage] * sm_count()));
    return launch_pdl(kern, dim3(grid), dim3(kMoeThreads), st, P);
}

template int launch_moe_fmt<QMV_FMT_ID>(int, const MoeParams&, int, cudaStream_t);
template int launch_mv_fmt<QMV_FMT_ID>(const MvParams&, int, cudaStream_t);
template int launch_sums_fmt<QMV_FMT_ID>(const MvParams&, cudaStream_t);
template int launch_tma_fmt<QMV_FMT_ID>(int, bool, const TmaParams&, const TmaPlan&, int, cudaStream_t);

}  // namespace qmv
