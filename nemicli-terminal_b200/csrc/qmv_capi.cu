// C ABI of the quantized matvec path (declarations and contracts: include/nemicli_qmv.h).
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <mutex>

#include "qmv_kernels.cuh"
#include "qmv_tma.cuh"
#include "qmv_chain.cuh"
#include "qmv_mma.cuh"
#include "../../include/nemicli_qmv.h"

using namespace qmv;

namespace {

thread_local int g_last_cuda_error = 0;
__device__ int g_device_status = 0;

// Workspace of qmv_chain_noalloc (barrier and group counters, activation buffers), for callers that
// cannot allocate.
static __device__ __align__(256) uint8_t g_chain_workspace[QMV_CHAIN_WORKSPACE_BYTES];
static_assert(QMV_CHAIN_NOALLOC_MAX_STAGES <= kChainMaxStages, "more stages than a chain takes");
static_assert(QMV_CHAIN_WORKSPACE_BYTES == kChainWorkspaceBytes, "workspace size in the header is stale");

// Address of g_chain_workspace on the current device, looked up once per device (with that device
// current) and cached; null if the lookup fails (its cudaError_t goes to qmv_last_cuda_error).
void* chain_workspace_ptr() {
    static std::mutex mu;
    static void* cache[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_chain_workspace);
        if (e != cudaSuccess || !p) {
            g_last_cuda_error = int(e);
            cudaGetLastError();                // do not leave the error for the next launch check
            return nullptr;
        }
        cache[dev] = p;
    }
    return cache[dev];
}

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

int launched() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_last_cuda_error = int(e);
        return ST_LAUNCH;
    }
    return ST_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int* device_status_ptr() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    return static_cast<int*>(p);
}

// common shape/pointer checks of a matvec call
int check_mv(int fmt, const void* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2, const float* xd,
             const float* xs, const void* y) {
    if (!known_format(fmt)) return ST_BAD_FORMAT;
    if (!w || !xq || !xq2 || !xd || !xs || !y) return ST_NULL;
    if (n_out <= 0 || n_in <= 0 || n_in % block_values(fmt)) return ST_BAD_SHAPE;
    if (!aligned(xq, 16) || !aligned(xq2, 16) || !aligned(xd, 8) || !aligned(xs, 8) || !aligned(y, 4))
        return ST_BAD_ALIGN;
    return ST_OK;
}

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

int launch(int fmt, const MvParams& P, int T, cudaStream_t st) {
    if (P.x_group < 1 || P.slots < 1) return ST_BAD_SHAPE;
    switch (fmt) {
    case F_Q4_0: return launch_fmt<F_Q4_0>(P, T, st);
    case F_Q8_0: return launch_fmt<F_Q8_0>(P, T, st);
    case F_Q4_K: return launch_fmt<F_Q4_K>(P, T, st);
    case F_Q5_K: return launch_fmt<F_Q5_K>(P, T, st);
    case F_Q6_K: return launch_fmt<F_Q6_K>(P, T, st);
    case F_IQ2_XXS: return launch_fmt<F_IQ2_XXS>(P, T, st);
    case F_TQ2_0: return launch_fmt<F_TQ2_0>(P, T, st);
    case F_IQ4_XS: return launch_fmt<F_IQ4_XS>(P, T, st);
    case F_MXFP4: return launch_fmt<F_MXFP4>(P, T, st);
    case F_IQ3_S: return launch_fmt<F_IQ3_S>(P, T, st);
    case F_IQ3_XXS: return launch_fmt<F_IQ3_XXS>(P, T, st);
    case F_Q4_1: return launch_fmt<F_Q4_1>(P, T, st);
    case F_Q5_0: return launch_fmt<F_Q5_0>(P, T, st);
    case F_Q5_1: return launch_fmt<F_Q5_1>(P, T, st);
    case F_IQ4_NL: return launch_fmt<F_IQ4_NL>(P, T, st);
    case F_Q1_0: return launch_fmt<F_Q1_0>(P, T, st);
    case F_Q2_0: return launch_fmt<F_Q2_0>(P, T, st);
    case F_PQ2_0: return launch_fmt<F_PQ2_0>(P, T, st);
    case F_Q3_K: return launch_fmt<F_Q3_K>(P, T, st);
    case F_Q2_K: return launch_fmt<F_Q2_K>(P, T, st);
    case F_TQ1_0: return launch_fmt<F_TQ1_0>(P, T, st);
    case F_IQ2_XS: return launch_fmt<F_IQ2_XS>(P, T, st);
    case F_IQ2_S: return launch_fmt<F_IQ2_S>(P, T, st);
    }
    return ST_BAD_FORMAT;
}

int launch_sums(int fmt, const MvParams& P, cudaStream_t st) {
    if (P.x_group != 1 || P.slots != 1) return ST_BAD_SHAPE;
    switch (fmt) {
    case F_Q4_0: return launch_t<F_Q4_0, 1, true>(P, st);
    case F_Q8_0: return launch_t<F_Q8_0, 1, true>(P, st);
    case F_Q4_K: return launch_t<F_Q4_K, 1, true>(P, st);
    case F_Q5_K: return launch_t<F_Q5_K, 1, true>(P, st);
    case F_Q6_K: return launch_t<F_Q6_K, 1, true>(P, st);
    case F_IQ2_XXS: return launch_t<F_IQ2_XXS, 1, true>(P, st);
    case F_TQ2_0: return launch_t<F_TQ2_0, 1, true>(P, st);
    case F_IQ4_XS: return launch_t<F_IQ4_XS, 1, true>(P, st);
    case F_MXFP4: return launch_t<F_MXFP4, 1, true>(P, st);
    case F_IQ3_S: return launch_t<F_IQ3_S, 1, true>(P, st);
    case F_IQ3_XXS: return launch_t<F_IQ3_XXS, 1, true>(P, st);
    case F_Q4_1: return launch_t<F_Q4_1, 1, true>(P, st);
    case F_Q5_0: return launch_t<F_Q5_0, 1, true>(P, st);
    case F_Q5_1: return launch_t<F_Q5_1, 1, true>(P, st);
    case F_IQ4_NL: return launch_t<F_IQ4_NL, 1, true>(P, st);
    case F_Q1_0: return launch_t<F_Q1_0, 1, true>(P, st);
    case F_Q2_0: return launch_t<F_Q2_0, 1, true>(P, st);
    case F_PQ2_0: return launch_t<F_PQ2_0, 1, true>(P, st);
    case F_Q3_K: return launch_t<F_Q3_K, 1, true>(P, st);
    case F_Q2_K: return launch_t<F_Q2_K, 1, true>(P, st);
    case F_TQ1_0: return launch_t<F_TQ1_0, 1, true>(P, st);
    case F_IQ2_XS: return launch_t<F_IQ2_XS, 1, true>(P, st);
    case F_IQ2_S: return launch_t<F_IQ2_S, 1, true>(P, st);
    }
    return ST_BAD_FORMAT;
}


// ---- TMA-staged single-token path ------------------------------------------------------------------

constexpr int kSmemCap = 232448;          // dynamic shared memory per block on sm_100a (227 KB)
constexpr int kSmemHalf = 113 * 1024;     // two CTAs per SM (the next kernel's CTA can prefetch alongside)
int g_pdl = 0;                            // programmatic dependent launch (qmv_set_pdl)

struct TmaPlan {
    int NCW, G, UPL, R, S, smem;
};

__host__ __device__ constexpr int unit_vals(int fmt) { return fmt == F_Q4_K || fmt == F_Q5_K || fmt == F_Q6_K ? 64 : 32; }   // UnitTraits::VPU

// Tuning knobs read once from the environment (benchmark sweeps): NEMICLI_QMV_TMA=0 sends every call
// to the fallback kernel, NEMICLI_QMV_TMA_G forces the team width (16..512) where it fits.
struct TmaKnobs {
    int enabled = 1, force_g = 0, ncw = 16;
    TmaKnobs() {
        if (const char* e = std::getenv("NEMICLI_QMV_TMA")) enabled = std::atoi(e) != 0;
        if (const char* g = std::getenv("NEMICLI_QMV_TMA_G")) force_g = std::atoi(g);
        if (const char* n = std::getenv("NEMICLI_QMV_NCW")) ncw = std::atoi(n) == 8 ? 8 : 16;
    }
};
const TmaKnobs& knobs() {
    static const TmaKnobs k;
    return k;
}

// Team width G (lanes per row), units per lane, rows per tile R = 4 rows per team (fewer when a stage
// would not fit twice), stages S; false if the shape needs the fallback kernel.  One unit per lane
// when a team of <= 512 lanes covers the row; fused quantisation reserves 2.25 * n_in bytes.
bool tma_plan(int fmt, int n_in, long long row_bytes, bool fused, TmaPlan& pl) {
    if (!knobs().enabled || row_bytes % 16 || n_in % unit_vals(fmt)) return false;
    if (fmt == F_TQ1_0) return false;          // TQ1_0 runs on the warp-per-row kernel only
    const int ncw = knobs().ncw;
    const int cap = ncw <= 8 ? kSmemHalf : kSmemCap;
    const int U = n_in / unit_vals(fmt);
    int G = 16;
    while (G < U && G < 32 * ncw) G *= 2;
    const int f = knobs().force_g;
    if (f >= 16 && f <= 32 * ncw && (f & (f - 1)) == 0 && 2 * f >= U) G = f;
    const int UPL = (U + G - 1) / G;
    if (UPL > 2) return false;
    const int teams = 32 * ncw / G;
    const long long other = tma_red_bytes(ncw) + 2048 + (fused ? tma_act_bytes(n_in) : 0) + 2 * 8 * 32;
    long long R = (long long)kTmaRowsPerTeam * teams;
    while (R > 1 && 2 * R * row_bytes > cap - other) R = R > teams ? R - teams : R / 2;
    const long long stage = R * row_bytes;
    long long S = (cap - other) / stage;
    if (S > 32) S = 32;
    if (S < 2) return false;
    pl.NCW = ncw;
    pl.G = G;
    pl.UPL = UPL;
    pl.R = int(R);
    pl.S = int(S);
    pl.smem = int(S * stage + other);
    return true;
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
    cfg.numAttrs = (g_pdl && !SUMS) ? 1 : 0;
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
int launch_tma_fmt(const TmaParams& P, const TmaPlan& pl, int grid, cudaStream_t st) {
    return pl.NCW == 16 ? launch_tma_g<FMT, 16, XF, SUMS>(P, pl, grid, st) : launch_tma_g<FMT, 8, XF, SUMS>(P, pl, grid, st);
}

template <int XF, bool SUMS>
int launch_tma(int fmt, TmaParams& P, const TmaPlan& pl, cudaStream_t st) {
    P.rows_per_tile = pl.R;
    P.stages = pl.S;
    P.status = device_status_ptr();
    long long grid = sm_count();
    if (grid > P.total_rows) grid = P.total_rows;
    if (grid < 1) return ST_OK;
    switch (fmt) {
    case F_Q4_0: return launch_tma_fmt<F_Q4_0, XF, SUMS>(P, pl, int(grid), st);
    case F_Q8_0: return launch_tma_fmt<F_Q8_0, XF, SUMS>(P, pl, int(grid), st);
    case F_Q4_K: return launch_tma_fmt<F_Q4_K, XF, SUMS>(P, pl, int(grid), st);
    case F_Q5_K: return launch_tma_fmt<F_Q5_K, XF, SUMS>(P, pl, int(grid), st);
    case F_Q6_K: return launch_tma_fmt<F_Q6_K, XF, SUMS>(P, pl, int(grid), st);
    case F_IQ2_XXS: return launch_tma_fmt<F_IQ2_XXS, XF, SUMS>(P, pl, int(grid), st);
    case F_TQ2_0: return launch_tma_fmt<F_TQ2_0, XF, SUMS>(P, pl, int(grid), st);
    case F_IQ4_XS: return launch_tma_fmt<F_IQ4_XS, XF, SUMS>(P, pl, int(grid), st);
    case F_MXFP4: return launch_tma_fmt<F_MXFP4, XF, SUMS>(P, pl, int(grid), st);
    case F_IQ3_S: return launch_tma_fmt<F_IQ3_S, XF, SUMS>(P, pl, int(grid), st);
    case F_IQ3_XXS: return launch_tma_fmt<F_IQ3_XXS, XF, SUMS>(P, pl, int(grid), st);
    case F_Q4_1: return launch_tma_fmt<F_Q4_1, XF, SUMS>(P, pl, int(grid), st);
    case F_Q5_0: return launch_tma_fmt<F_Q5_0, XF, SUMS>(P, pl, int(grid), st);
    case F_Q5_1: return launch_tma_fmt<F_Q5_1, XF, SUMS>(P, pl, int(grid), st);
    case F_IQ4_NL: return launch_tma_fmt<F_IQ4_NL, XF, SUMS>(P, pl, int(grid), st);
    case F_Q1_0: return launch_tma_fmt<F_Q1_0, XF, SUMS>(P, pl, int(grid), st);
    case F_Q2_0: return launch_tma_fmt<F_Q2_0, XF, SUMS>(P, pl, int(grid), st);
    case F_PQ2_0: return launch_tma_fmt<F_PQ2_0, XF, SUMS>(P, pl, int(grid), st);
    case F_Q3_K: return launch_tma_fmt<F_Q3_K, XF, SUMS>(P, pl, int(grid), st);
    case F_Q2_K: return launch_tma_fmt<F_Q2_K, XF, SUMS>(P, pl, int(grid), st);
    case F_IQ2_XS: return launch_tma_fmt<F_IQ2_XS, XF, SUMS>(P, pl, int(grid), st);
    case F_IQ2_S: return launch_tma_fmt<F_IQ2_S, XF, SUMS>(P, pl, int(grid), st);
    }
    return ST_BAD_FORMAT;
}

// dense jobs sharing one activation row (n_jobs <= kMaxJobs): pre-quantised (x == nullptr) or raw x
// (x_kind 1 = fp32, 2 = bf16) quantised in the kernel.  false -> the caller uses the fallback kernel.
bool tma_dense(int fmt, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
               const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, const void* x, int x_kind,
               int32_t* s, int32_t* s2, cudaStream_t st, int* status) {
    const long long row_bytes = (long long)(n_in / block_values(fmt)) * block_bytes(fmt);
    TmaPlan pl;
    if (!tma_plan(fmt, n_in, row_bytes, x != nullptr, pl)) return false;
    for (int j = 0; j < n_jobs; ++j)
        if (!aligned(w[j], 16)) return false;
    TmaParams P{};
    long long rows = 0;
    for (int j = 0; j < n_jobs; ++j) {
        P.w[j] = w[j];
        P.y[j] = y ? y[j] : nullptr;
        P.n_out[j] = n_out[j];
        P.row_start[j] = rows;
        rows += n_out[j];
    }
    P.row_start[n_jobs] = rows;
    P.n_jobs = n_jobs;
    P.x_group = 1;
    P.xq = xq; P.xq2 = xq2; P.xd = xd; P.xs = xs;
    P.x = x;
    P.row_bytes = row_bytes;
    P.n_in = n_in;
    P.total_rows = rows;
    P.s = s; P.s2 = s2;
    if (s) *status = launch_tma<0, true>(fmt, P, pl, st);
    else if (!x) *status = launch_tma<0, false>(fmt, P, pl, st);
    else if (x_kind == 1) *status = launch_tma<1, false>(fmt, P, pl, st);
    else *status = launch_tma<2, false>(fmt, P, pl, st);
    return true;
}

}  // namespace

namespace {
// Few-token Q4_K / Q8_0 matvec on the tensor cores; false when the shape or alignment does not qualify.
template <int FMT>
bool mma_dense_k(const uint8_t* w, int n_out, int n_in, long long row_bytes, const int8_t* xq, const int8_t* xq2,
                 const float* xd, const float* xs, int T, float* y, cudaStream_t st, int* status) {
    if (T < 2 || T > kMmaMaxTok || n_in % block_values(FMT) || n_in > kMmaMaxIn || !knobs().enabled) return false;
    if (!aligned(w, 16) || !aligned(xq, 16) || !aligned(xq2, 16) || row_bytes % 16) return false;
    constexpr int NCW = 16;
    const long long other = mma_act_bytes(n_in) + mma_red_bytes(NCW) + 2 * 8 * 32;
    const long long slot = kMmaRows * mma_row_stride(row_bytes);
    long long S = (kSmemCap - other) / slot;
    if (S > 4) S = 4;
    if (S < 2) return false;
    MmaParams P{};
    P.w = w; P.y = y; P.xq = xq; P.xq2 = xq2; P.xd = xd; P.xs = xs;
    P.row_bytes = row_bytes; P.n_out = n_out; P.n_in = n_in; P.n_tok = T; P.stages = int(S);
    P.status = device_status_ptr();
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(mv_mma_kernel<FMT, NCW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess) {
            *status = launched();
            return true;
        }
        configured[dev] = 1;
    }
    const int tiles = (n_out + kMmaRows - 1) / kMmaRows;
    const int grid = std::min(tiles, sm_count());
    mv_mma_kernel<FMT, NCW><<<grid, 32 * (NCW + 1), int(S * slot + other), st>>>(P);
    *status = launched();
    return true;
}
bool mma_q4k(const uint8_t* w, int n_out, int n_in, long long row_bytes, const int8_t* xq, const int8_t* xq2,
             const float* xd, const float* xs, int T, float* y, int fmt, cudaStream_t st, int* status) {
    if (fmt == F_Q4_K) return mma_dense_k<F_Q4_K>(w, n_out, n_in, row_bytes, xq, xq2, xd, xs, T, y, st, status);
    if (fmt == F_Q8_0) return mma_dense_k<F_Q8_0>(w, n_out, n_in, row_bytes, xq, xq2, xd, xs, T, y, st, status);
    return false;
}

// Few-token Q6_K matvec on the tensor cores (rows of a multiple of 2048 values).
bool mma_q6k(const uint8_t* w, int n_out, int n_in, long long row_bytes, const int8_t* xq, const int8_t* xq2,
             const float* xd, int T, float* y, int fmt, cudaStream_t st, int* status) {
    if (fmt != F_Q6_K || T < 2 || T > kMmaMaxTok || n_in % kQ6Chunk || !knobs().enabled) return false;
    if (!aligned(w, 16) || !aligned(xq, 16) || !aligned(xq2, 16) || row_bytes % 16) return false;
    constexpr int NCW = 16;
    const int n_rb = (n_out + kMmaRows - 1) / kMmaRows;
    const int grid = std::min(n_rb, sm_count());
    if ((n_rb + grid - 1) / grid > kQ6MaxBlocks) return false;
    if (!aligned(xd, 16)) return false;
    const long long other = 2LL * kQ6ActBytes + mma_red_bytes(NCW) + 4LL * kQ6MaxBlocks * kMmaRows * kMmaMaxTok + 2 * 8 * 32;
    const long long slot = (long long)kMmaRows * kQ6ChunkBytes;
    long long S = (kSmemCap - other) / slot;
    if (S > 6) S = 6;
    if (S < 2) return false;
    MmaParams P{};
    P.w = w; P.y = y; P.xq = xq; P.xq2 = xq2; P.xd = xd; P.xs = nullptr;
    P.row_bytes = row_bytes; P.n_out = n_out; P.n_in = n_in; P.n_tok = T; P.stages = int(S);
    P.status = device_status_ptr();
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(mv_mma_q6k_kernel<NCW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess) {
            *status = launched();
            return true;
        }
        configured[dev] = 1;
    }
    mv_mma_q6k_kernel<NCW><<<grid, 32 * (NCW + 1), int(S * slot + other), st>>>(P);
    *status = launched();
    return true;
}
}  // namespace

extern "C" {

int qmv_abi_version(void) { return NEMICLI_QMV_ABI_VERSION; }

const char* qmv_status_string(int status) {
    switch (status) {
    case ST_OK: return "ok";
    case ST_BAD_FORMAT: return "unsupported block format";
    case ST_BAD_SHAPE: return "bad shape (n_in must be a positive multiple of the block size, n_out > 0)";
    case ST_BAD_ALIGN: return "misaligned pointer";
    case ST_BAD_TOKENS: return "token count out of range";
    case ST_LAUNCH: return "CUDA launch failed";
    case ST_NULL: return "null pointer";
    case ST_DEVICE: return "device status query failed";
    case QMV_ERR_TOO_LARGE: return "size beyond the fixed maximum of a no-allocation entry point";
    }
    return "unknown status";
}

int qmv_last_cuda_error(void) { return g_last_cuda_error; }

int qmv_block_values(int ggml_type) { return known_format(ggml_type) ? block_values(ggml_type) : 0; }
int qmv_block_bytes(int ggml_type) { return known_format(ggml_type) ? block_bytes(ggml_type) : 0; }

int qmv_supported(int ggml_type, int n_in) {
    return known_format(ggml_type) && n_in > 0 && n_in % block_values(ggml_type) == 0;
}

int qmv_quant_q8(const void* x, int x_is_f32, int8_t* xq, int8_t* xq2, float* xd, float* xs, long long n,
                 void* stream) {
    if (!x || !xq || !xq2 || !xd || !xs) return ST_NULL;
    if (n <= 0 || n % 32) return ST_BAD_SHAPE;
    if (!aligned(x, x_is_f32 ? 4 : 2)) return ST_BAD_ALIGN;
    const long long blocks = (n + 255) / 256;
    quant_q8_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, x_is_f32, xq, xq2, xd, xs, n);
    return launched();
}

int qmv_mv(int ggml_type, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
           const float* xd, const float* xs, int n_tok, float* y, void* stream) {
    int st = check_mv(ggml_type, w, n_out, n_in, xq, xq2, xd, xs, y);
    if (st) return st;
    if (n_tok <= 0) return ST_BAD_TOKENS;
    if (!aligned(w, weight_align(ggml_type))) return ST_BAD_ALIGN;
    MvParams P{};
    P.w = w;
    P.ids = nullptr;
    P.per_expert = 0;
    P.row_bytes = (long long)(n_in / block_values(ggml_type)) * block_bytes(ggml_type);
    P.x_group = 1;
    P.status = device_status_ptr();
    P.n_out = n_out;
    P.n_in = n_in;
    P.slots = 1;
    if (n_tok == 1) {
        float* ys[1] = {y};
        const uint8_t* ws[1] = {w};
        const int nos[1] = {n_out};
        if (tma_dense(ggml_type, 1, ws, nos, ys, n_in, xq, xq2, xd, xs, nullptr, 0, nullptr, nullptr,
                      static_cast<cudaStream_t>(stream), &st))
            return st;
    }
    for (int c0 = 0; c0 < n_tok; c0 += kMaxTokens) {
        const int T = n_tok - c0 < kMaxTokens ? n_tok - c0 : kMaxTokens;
        const long long off = (long long)c0 * n_in;
        // 2..8 tokens of Q4_K / Q8_0 rows up to kMmaMaxIn values, or of Q6_K rows: the tensor-core kernels
        if (T >= 2 && (mma_q4k(w, n_out, n_in, P.row_bytes, xq + off, xq2 + off, xd + off / 32, xs + off / 32, T,
                               y + (long long)c0 * n_out, ggml_type, static_cast<cudaStream_t>(stream), &st) ||
                       mma_q6k(w, n_out, n_in, P.row_bytes, xq + off, xq2 + off, xd + off / 32, T,
                               y + (long long)c0 * n_out, ggml_type, static_cast<cudaStream_t>(stream), &st))) {
            if (st) return st;
            continue;
        }
        P.xq = xq + off;
        P.xq2 = xq2 + off;
        P.xd = xd + off / 32;
        P.xs = xs + off / 32;
        P.y = y + (long long)c0 * n_out;
        if ((st = launch(ggml_type, P, T, static_cast<cudaStream_t>(stream)))) return st;
    }
    return ST_OK;
}

int qmv_mv_experts(int ggml_type, const void* raw, long long per_expert, long long n_exp, const long long* ids, int k,
                   const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int x_group,
                   float* y, int n_out, int n_in, void* stream) {
    int st = check_mv(ggml_type, raw, n_out, n_in, xq, xq2, xd, xs, y);
    if (st) return st;
    if (!ids) return ST_NULL;
    if (k <= 0) return ST_BAD_TOKENS;
    if (n_exp <= 0) return ST_BAD_SHAPE;
    if (x_group <= 0) return ST_BAD_SHAPE;
    const long long row_bytes = (long long)(n_in / block_values(ggml_type)) * block_bytes(ggml_type);
    if (per_expert >= 0) {
        if (per_expert < row_bytes * n_out) return ST_BAD_SHAPE;
        if (!aligned(raw, weight_align(ggml_type)) || per_expert % (weight_align(ggml_type)))
            return ST_BAD_ALIGN;
    } else if (!aligned(raw, 8)) {
        return ST_BAD_ALIGN;
    }
    MvParams P{};
    P.w = static_cast<const uint8_t*>(raw);
    P.ids = ids;
    P.per_expert = per_expert >= 0 ? per_expert : -1;
    P.row_bytes = row_bytes;
    P.xq = xq;
    P.xq2 = xq2;
    P.xd = xd;
    P.xs = xs;
    P.x_group = x_group;
    P.y = y;
    P.status = device_status_ptr();
    P.n_out = n_out;
    P.n_in = n_in;
    P.slots = k;
    P.n_exp = n_exp;
    TmaPlan pl;
    if (tma_plan(ggml_type, n_in, row_bytes, false, pl) && aligned(raw, 16) && (per_expert < 0 || per_expert % 16 == 0)) {
        TmaParams Q{};
        Q.w[0] = static_cast<const uint8_t*>(raw);
        Q.y[0] = y;
        Q.n_out[0] = n_out;
        Q.n_jobs = 1;
        Q.ids = ids;
        Q.per_expert = per_expert >= 0 ? per_expert : -1;
        Q.n_exp = n_exp;
        Q.x_group = x_group;
        Q.xq = xq; Q.xq2 = xq2; Q.xd = xd; Q.xs = xs;
        Q.row_bytes = row_bytes;
        Q.n_in = n_in;
        Q.total_rows = (long long)n_out * k;
        return launch_tma<0, false>(ggml_type, Q, pl, static_cast<cudaStream_t>(stream));
    }
    return launch(ggml_type, P, 1, static_cast<cudaStream_t>(stream));
}

int qmv_block_sums(int ggml_type, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
                   int32_t* s, int32_t* s2, void* stream) {
    if (!known_format(ggml_type)) return ST_BAD_FORMAT;
    if (!w || !xq || !xq2 || !s || !s2) return ST_NULL;
    if (n_out <= 0 || n_in <= 0 || n_in % block_values(ggml_type)) return ST_BAD_SHAPE;
    if (!aligned(xq, 16) || !aligned(xq2, 16) || !aligned(s, 4) || !aligned(s2, 4)) return ST_BAD_ALIGN;
    if (!aligned(w, weight_align(ggml_type))) return ST_BAD_ALIGN;
    const long long units = (long long)n_out * (n_in / unit_values(ggml_type));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(s, 0, units * sizeof(int32_t), st) != cudaSuccess ||
        cudaMemsetAsync(s2, 0, units * sizeof(int32_t), st) != cudaSuccess) {
        g_last_cuda_error = int(cudaGetLastError());
        return ST_LAUNCH;
    }
    {
        const uint8_t* ws[1] = {w};
        const int nos[1] = {n_out};
        int rc = ST_OK;
        if (tma_dense(ggml_type, 1, ws, nos, nullptr, n_in, xq, xq2, nullptr, nullptr, nullptr, 0, s, s2, st, &rc))
            return rc;
    }
    MvParams P{};
    P.w = w;
    P.row_bytes = (long long)(n_in / block_values(ggml_type)) * block_bytes(ggml_type);
    P.xq = xq;
    P.xq2 = xq2;
    P.s = s;
    P.s2 = s2;
    P.x_group = 1;
    P.status = device_status_ptr();
    P.n_out = n_out;
    P.n_in = n_in;
    P.slots = 1;
    return launch_sums(ggml_type, P, st);
}

int qmv_mv_multi(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                 const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, void* stream) {
    if (!w || !n_out || !y) return ST_NULL;
    if (n_jobs < 1 || n_jobs > kMaxJobs) return ST_BAD_TOKENS;
    for (int j = 0; j < n_jobs; ++j) {
        const int st = check_mv(ggml_type, w[j], n_out[j], n_in, xq, xq2, xd, xs, y[j]);
        if (st) return st;
        if (!aligned(w[j], weight_align(ggml_type))) return ST_BAD_ALIGN;
    }
    int st = ST_OK;
    if (tma_dense(ggml_type, n_jobs, w, n_out, y, n_in, xq, xq2, xd, xs, nullptr, 0, nullptr, nullptr,
                  static_cast<cudaStream_t>(stream), &st))
        return st;
    for (int j = 0; j < n_jobs; ++j)
        if ((st = qmv_mv(ggml_type, w[j], n_out[j], n_in, xq, xq2, xd, xs, 1, y[j], stream))) return st;
    return ST_OK;
}

int qmv_mv_x(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
             const void* x, int x_is_f32, void* stream) {
    if (!w || !n_out || !y || !x) return ST_NULL;
    if (!known_format(ggml_type)) return ST_BAD_FORMAT;
    if (n_jobs < 1 || n_jobs > kMaxJobs) return ST_BAD_TOKENS;
    if (n_in <= 0 || n_in % block_values(ggml_type)) return ST_BAD_SHAPE;
    if (!aligned(x, x_is_f32 ? 4 : 2)) return ST_BAD_ALIGN;
    for (int j = 0; j < n_jobs; ++j) {
        if (!w[j] || !y[j]) return ST_NULL;
        if (n_out[j] <= 0) return ST_BAD_SHAPE;
        if (!aligned(w[j], weight_align(ggml_type)) || !aligned(y[j], 4)) return ST_BAD_ALIGN;
    }
    int st = ST_OK;
    if (tma_dense(ggml_type, n_jobs, w, n_out, y, n_in, nullptr, nullptr, nullptr, nullptr, x, x_is_f32 ? 1 : 2,
                  nullptr, nullptr, static_cast<cudaStream_t>(stream), &st))
        return st;
    return ST_BAD_SHAPE;        // the shape needs the fallback kernel: quantise with qmv_quant_q8, then qmv_mv
}

int qmv_chain(const qmv_stage* stages, int n_stages, void* workspace, void* stream) {
    if (!stages || !workspace) return ST_NULL;
    if (n_stages < 1 || n_stages > kChainMaxStages) return ST_BAD_TOKENS;
    if (!aligned(workspace, 256)) return ST_BAD_ALIGN;
    static ChainParams P;                     // host staging of the kernel parameters (~25 KB)
    static std::mutex mu;
    std::lock_guard<std::mutex> lock(mu);
    P = ChainParams{};
    long long slot = 0;
    for (int k = 0; k < n_stages; ++k) {
        const qmv_stage& q = stages[k];
        ChainStage& c = P.st[k];
        int cfg = -1;
        if (q.ggml_type == F_Q4_K && q.n_in == 4096) cfg = CFG_Q4K_4096;
        else if (q.ggml_type == F_Q6_K && q.n_in == 14336) cfg = CFG_Q6K_14336;
        else if (q.ggml_type == F_Q4_K && q.n_in == 14336) cfg = CFG_Q4K_14336;
        else if (q.ggml_type == F_Q6_K && q.n_in == 4096) cfg = CFG_Q6K_4096;
        else if (q.ggml_type == F_Q8_0 && q.n_in == 4096) cfg = CFG_Q8_0_4096;
        if (cfg < 0) return known_format(q.ggml_type) ? ST_BAD_SHAPE : ST_BAD_FORMAT;
        if (q.n_jobs < 1 || q.n_jobs > kMaxJobs) return ST_BAD_TOKENS;
        if (!q.a || (q.input == QMV_INPUT_RMSNORM && !q.norm_w)) return ST_NULL;
        if (q.input < 0 || q.input > 2) return ST_BAD_SHAPE;
        if (!aligned(q.a, 4) || (q.b && !aligned(q.b, 4))) return ST_BAD_ALIGN;
        c.cfg = cfg;
        c.n_jobs = q.n_jobs;
        c.n_in = q.n_in;
        c.row_bytes = (long long)(q.n_in / block_values(q.ggml_type)) * block_bytes(q.ggml_type);
        long long rows = 0;
        for (int j = 0; j < q.n_jobs; ++j) {
            if (!q.w[j] || !q.y[j]) return ST_NULL;
            if (q.n_out[j] <= 0) return ST_BAD_SHAPE;
            if (!aligned(q.w[j], 16) || !aligned(q.y[j], 4)) return ST_BAD_ALIGN;
            c.w[j] = q.w[j];
            c.y[j] = q.y[j];
            c.n_out[j] = q.n_out[j];
            c.row_start[j] = rows;
            rows += q.n_out[j];
        }
        c.row_start[q.n_jobs] = rows;
        c.total_rows = rows;
        c.R = chain_cfg_nper(cfg) * (32 * kChainNcw / chain_cfg_g(cfg));
        c.in_kind = q.input;
        c.a = q.a;
        c.b = q.input == QMV_INPUT_RAW ? nullptr : q.b;
        c.norm_w = q.norm_w;
        c.eps = q.eps;
        c.h_out = q.h_out;
        c.wait = k > 0 && q.wait;
        slot = std::max(slot, (long long)c.R * c.row_bytes);
    }
    // fed stages: every input vector that the previous stage writes is one whole job output of it; the
    // previous stage's CTAs then quantise the input group by group as they complete it
    for (int k = 1; k < n_stages; ++k) {
        ChainStage& c = P.st[k];
        ChainStage& pv = P.st[k - 1];
        if (!c.wait) continue;
        auto job_of = [&](const float* v) -> int {
            for (int j = 0; j < pv.n_jobs; ++j)
                if (v && pv.y[j] == v && pv.n_out[j] == c.n_in) return j;
            return -1;
        };
        const int ja = job_of(c.a), jb = job_of(c.b);
        bool ok = false;
        if (c.in_kind == CH_RAW) ok = ja >= 0;
        else if (c.in_kind == CH_SILU_MUL) ok = ja >= 0 && (c.b == nullptr || jb >= 0);
        else ok = ja >= 0 || jb >= 0;
        if (!ok) continue;
        const int mask = (ja >= 0 ? 1 << ja : 0) | (jb >= 0 ? 1 << jb : 0);
        c.fed = 1;
        pv.feed_mask = mask;
        pv.feed_target = 32 * __builtin_popcount(mask);
    }
    // the kernel instance that carries every configuration this chain uses (at most two)
    int used = 0;
    for (int k = 0; k < n_stages; ++k) used |= 1 << P.st[k].cfg;
    const int pairs[4][2] = {{CFG_Q4K_4096, CFG_Q6K_14336}, {CFG_Q4K_4096, CFG_Q4K_14336},
                             {CFG_Q6K_4096, CFG_Q6K_14336}, {CFG_Q8_0_4096, CFG_Q6K_4096}};
    int pair = -1;
    for (int i = 0; i < 4 && pair < 0; ++i)
        if ((used & ~((1 << pairs[i][0]) | (1 << pairs[i][1]))) == 0) pair = i;
    if (pair < 0) return ST_BAD_SHAPE;           // more than two row shapes: split the chain
    slot = (slot + 127) / 128 * 128;
    const long long other = chain_red_bytes() + 2 * 8 * 32;
    long long S = (kSmemCap - other) / slot;
    // three slots: deeper rings only add queueing latency to every other memory access (measured)
    static const int env_slots = getenv("NEMICLI_CHAIN_SLOTS") ? atoi(getenv("NEMICLI_CHAIN_SLOTS")) : 3;
    if (env_slots >= 2 && env_slots < S) S = env_slots;
    if (S > 32) S = 32;
    if (S < 2) return ST_BAD_SHAPE;
    P.n_stages = n_stages;
    P.S = int(S);
    P.slot_bytes = int(slot);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    P.bar = reinterpret_cast<int*>(ws);
    P.cnt = P.bar + 2 * kChainMaxStages;
    for (int b = 0; b < 2; ++b) {
        uint8_t* base = ws + kChainCounterBytes + b * kChainActBytes;
        P.xq[b] = reinterpret_cast<int8_t*>(base);
        P.xq2[b] = P.xq[b] + kChainMaxIn;
        P.xd[b] = reinterpret_cast<float*>(P.xq2[b] + kChainMaxIn);
        P.xs[b] = P.xd[b] + kChainMaxGroups;
        P.pss[b] = P.xs[b] + kChainMaxGroups;
    }
    P.status = device_status_ptr();
    const int smem = int(S * slot + other);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(workspace, 0, kChainCounterBytes, st) != cudaSuccess) return launched();
    void (*kern)(const ChainParams) = pair == 0 ? chain_kernel<kChainNcw, CFG_Q4K_4096, CFG_Q6K_14336>
                                    : pair == 1 ? chain_kernel<kChainNcw, CFG_Q4K_4096, CFG_Q4K_14336>
                                    : pair == 2 ? chain_kernel<kChainNcw, CFG_Q6K_4096, CFG_Q6K_14336>
                                                : chain_kernel<kChainNcw, CFG_Q8_0_4096, CFG_Q6K_4096>;
    static int configured[64][4] = {{0}};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev][pair]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess)
            return launched();
        configured[dev][pair] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count());
    cfg.blockDim = dim3(32 * (kChainNcw + 1));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, kern, P) != cudaSuccess) return launched();
    return launched();
}

int64_t qmv_chain_workspace_bytes(void) { return kChainWorkspaceBytes; }

int qmv_chain_noalloc(const qmv_stage* stages, int n_stages, void* stream) {
    if (!stages) return ST_NULL;
    if (n_stages > QMV_CHAIN_NOALLOC_MAX_STAGES) return QMV_ERR_TOO_LARGE;
    if (n_stages < 1) return ST_BAD_TOKENS;
    void* ws = chain_workspace_ptr();
    if (!ws) return ST_DEVICE;
    return qmv_chain(stages, n_stages, ws, stream);           // clears the counters on `stream`
}

int qmv_set_pdl(int enabled) {
    const int old = g_pdl;
    g_pdl = enabled ? 1 : 0;
    return old;
}

int qmv_device_status(int clear, int* out, void* stream) {
    if (!out) return ST_NULL;
    int* p = device_status_ptr();
    if (!p) return ST_DEVICE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(out, p, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return ST_DEVICE;
    if (cudaStreamSynchronize(st) != cudaSuccess) return ST_DEVICE;
    if (clear && cudaMemsetAsync(p, 0, sizeof(int), st) != cudaSuccess) return ST_DEVICE;
    return ST_OK;
}

}  // extern "C"
