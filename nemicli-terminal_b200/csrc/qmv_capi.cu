// C ABI of the quantized matvec path (declarations and contracts: include/nemicli_qmv.h).  The kernels
// themselves are instantiated in the other translation units (qmv_host.cuh lists them); this file checks
// arguments, plans the launch and dispatches by format.  The decode chain's entry points are in qmv_chain.cu.
#include <cstdio>
#include <cstdlib>
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "qmv_host.cuh"
#include "qmv_moe.cuh"
#include "../../include/nemicli_qmv.h"

using namespace qmv;

namespace {

thread_local int g_last_cuda_error = 0;
__device__ int g_device_status = 0;
int g_pdl = 0;                            // programmatic dependent launch (qmv_set_pdl)

// Kernel geometry.  The shipped library uses the fixed values below; a build with -DQMV_SWEEP (benchmark
// sweeps only, never the shipped library) reads them once from the environment: NEMICLI_QMV_TMA=0 sends
// every call to the fallback kernel, NEMICLI_QMV_TMA_G forces the team width (16..512) where it fits.
struct TmaKnobs {
    int enabled = 1, force_g = 0, ncw = 16, rows_per_team = kTmaRowsPerTeam;
    TmaKnobs() {
#ifdef QMV_SWEEP
        if (const char* e = std::getenv("NEMICLI_QMV_ROWS")) rows_per_team = std::max(1, std::min(4, std::atoi(e)));
        if (const char* e = std::getenv("NEMICLI_QMV_TMA")) enabled = std::atoi(e) != 0;
        if (const char* g = std::getenv("NEMICLI_QMV_TMA_G")) force_g = std::atoi(g);
        if (const char* n = std::getenv("NEMICLI_QMV_NCW")) ncw = std::atoi(n) == 8 ? 8 : 16;
#endif
    }
};
const TmaKnobs& knobs() {
    static const TmaKnobs k;
    return k;
}

}  // namespace

namespace qmv {

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

void set_last_cuda_error(int e) { g_last_cuda_error = e; }

int launched() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_last_cuda_error = int(e);
        return ST_LAUNCH;
    }
    return ST_OK;
}

int* device_status_ptr() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    return static_cast<int*>(p);
}

bool pdl_enabled() { return g_pdl != 0; }
bool tma_enabled() { return knobs().enabled != 0; }

}  // namespace qmv

namespace {

// Calls f(std::integral_constant<int, FMT>) for the format id fmt; ST_BAD_FORMAT for an unknown id.
template <class Fn>
int by_format(int fmt, Fn&& f) {
#define QMV_CASE(F) case F: return f(std::integral_constant<int, F>{});
    switch (fmt) {
    QMV_CASE(F_Q4_0) QMV_CASE(F_Q4_1) QMV_CASE(F_Q5_0) QMV_CASE(F_Q5_1) QMV_CASE(F_Q8_0) QMV_CASE(F_IQ4_NL)
    QMV_CASE(F_MXFP4) QMV_CASE(F_Q1_0) QMV_CASE(F_Q2_0) QMV_CASE(F_PQ2_0) QMV_CASE(F_Q2_K) QMV_CASE(F_Q3_K)
    QMV_CASE(F_Q4_K) QMV_CASE(F_Q5_K) QMV_CASE(F_Q6_K) QMV_CASE(F_IQ2_XXS) QMV_CASE(F_IQ2_XS) QMV_CASE(F_IQ2_S)
    QMV_CASE(F_IQ3_XXS) QMV_CASE(F_IQ3_S) QMV_CASE(F_IQ4_XS) QMV_CASE(F_TQ1_0) QMV_CASE(F_TQ2_0)
    QMV_CASE(F_IQ1_S) QMV_CASE(F_IQ1_M) QMV_CASE(F_PTQ1_0)
    }
#undef QMV_CASE
    return ST_BAD_FORMAT;
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

int launch(int fmt, const MvParams& P, int T, cudaStream_t st) {
    if (P.x_group < 1 || P.slots < 1) return ST_BAD_SHAPE;
    return by_format(fmt, [&](auto c) { return launch_mv_fmt<decltype(c)::value>(P, T, st); });
}

int launch_sums(int fmt, const MvParams& P, cudaStream_t st) {
    if (P.x_group != 1 || P.slots != 1) return ST_BAD_SHAPE;
    return by_format(fmt, [&](auto c) { return launch_sums_fmt<decltype(c)::value>(P, st); });
}

// ---- TMA-staged single-token path ------------------------------------------------------------------

__host__ __device__ constexpr int unit_vals(int fmt) { return fmt == F_Q4_K || fmt == F_Q5_K || fmt == F_Q6_K ? 64 : 32; }   // UnitTraits::VPU

// Team width G (lanes per row), units per lane, rows per tile R = 4 rows per team (fewer when a stage
// would not fit twice), stages S; false if the shape needs the fallback kernel.  One unit per lane
// when a team of <= 512 lanes covers the row; fused quantisation reserves 2.25 * n_in bytes.
bool tma_plan(int fmt, int n_in, long long row_bytes, bool fused, TmaPlan& pl) {
    if (!knobs().enabled || row_bytes % 16 || n_in % unit_vals(fmt)) return false;
    if (!staged_format(fmt)) return false;     // TQ1_0, IQ1_S, IQ1_M, PTQ1_0 run on the warp-per-row kernel only
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
    long long R = (long long)knobs().rows_per_team * teams;
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

template <int XF, bool SUMS>
int launch_tma(int fmt, TmaParams& P, const TmaPlan& pl, cudaStream_t st) {
    P.rows_per_tile = pl.R;
    P.stages = pl.S;
    P.status = device_status_ptr();
    long long grid = sm_count();
    if (grid > P.total_rows) grid = P.total_rows;
    if (grid < 1) return ST_OK;
    return by_format(fmt, [&](auto c) { return launch_tma_fmt<decltype(c)::value>(XF, SUMS, P, pl, int(grid), st); });
}

// dense jobs sharing one activation row (n_jobs <= kMaxJobs): pre-quantised (x == nullptr) or raw x
// (x_kind 1 = fp32, 2 = bf16) quantised in the kernel.  false -> the caller uses the fallback kernel.
struct EpOut {                   // epilogue producer (TmaParams ep_*)
    int kind, j0, j1;
    int* cnt;
    int8_t* xq;
    int8_t* xq2;
    float* xd;
    float* xs;
    float* a;
};

struct NormIn {                  // fused RMS norm of an fp32 x (TmaParams nr .. neps)
    const float* r;
    float rs;
    float* h_out;
    const float* w;
    float eps;
};

bool tma_dense(int fmt, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
               const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, const void* x, int x_kind,
               int32_t* s, int32_t* s2, cudaStream_t st, int* status, const NormIn* norm = nullptr,
               const EpOut* ep = nullptr) {
    const long long row_bytes = (long long)(n_in / block_values(fmt)) * block_bytes(fmt);
    TmaPlan pl;
    if (!tma_plan(fmt, n_in, row_bytes, x != nullptr, pl)) return false;
    if (ep && pl.G <= 32) return false;          // the epilogue runs in the wide teams' window flush
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
    if (norm) {
        P.nr = norm->r; P.nrs = norm->rs; P.nh = norm->h_out; P.nw = norm->w; P.neps = norm->eps;
    }
    if (ep) {
        P.ep_kind = ep->kind; P.ep_j0 = ep->j0; P.ep_j1 = ep->j1; P.ep_cnt = ep->cnt;
        P.ep_xq = ep->xq; P.ep_xq2 = ep->xq2; P.ep_xd = ep->xd; P.ep_xs = ep->xs; P.ep_a = ep->a;
    }
    if (s) *status = launch_tma<0, true>(fmt, P, pl, st);
    else if (!x) *status = launch_tma<0, false>(fmt, P, pl, st);
    else if (x_kind == 1) *status = launch_tma<1, false>(fmt, P, pl, st);
    else *status = launch_tma<2, false>(fmt, P, pl, st);
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

int qmv_unit_values(int ggml_type) { return known_format(ggml_type) ? unit_values(ggml_type) : 0; }

int qmv_supported(int ggml_type, int n_in) {
    return known_format(ggml_type) && n_in > 0 && n_in % block_values(ggml_type) == 0;
}

int qmv_quant_q8(const void* x, int x_is_f32, int8_t* xq, int8_t* xq2, float* xd, float* xs, long long n,
                 void* stream) {
    if (!x || !xq || !xq2 || !xd || !xs) return ST_NULL;
    if (n <= 0 || n % 32) return ST_BAD_SHAPE;
    if (!aligned(x, x_is_f32 ? 4 : 2)) return ST_BAD_ALIGN;
    const long long blocks = (n + 255) / 256;
    return launch_pdl(quant_q8_kernel, dim3(unsigned(blocks)), dim3(256), static_cast<cudaStream_t>(stream), x,
                      x_is_f32, xq, xq2, xd, xs, n);
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

int qmv_mv_multi_tok(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                     const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int n_tok, void* stream) {
    if (!w || !n_out || !y) return ST_NULL;
    if (n_jobs < 1 || n_jobs > kMaxJobs || n_tok <= 0) return ST_BAD_TOKENS;
    if (n_tok == 1) return qmv_mv_multi(ggml_type, n_jobs, w, n_out, y, n_in, xq, xq2, xd, xs, stream);
    for (int j = 0; j < n_jobs; ++j) {
        const int st = check_mv(ggml_type, w[j], n_out[j], n_in, xq, xq2, xd, xs, y[j]);
        if (st) return st;
        if (!aligned(w[j], weight_align(ggml_type))) return ST_BAD_ALIGN;
    }
    const long long row_bytes = (long long)(n_in / block_values(ggml_type)) * block_bytes(ggml_type);
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    for (int c0 = 0; c0 < n_tok; c0 += kMaxTokens) {         // groups of up to 8 tokens
        const int T = n_tok - c0 < kMaxTokens ? n_tok - c0 : kMaxTokens;
        const long long off = (long long)c0 * n_in;
        float* yc[kMaxJobs];
        for (int j = 0; j < n_jobs; ++j) yc[j] = y[j] + (long long)c0 * n_out[j];
        int st = ST_OK;
        if (T >= 2 &&
            mma_q4k_multi(n_jobs, w, n_out, yc, n_in, row_bytes, xq + off, xq2 + off, xd + off / 32, xs + off / 32, T,
                          ggml_type, cs, &st)) {
            if (st) return st;
            continue;
        }
        for (int j = 0; j < n_jobs; ++j)
            if ((st = qmv_mv(ggml_type, w[j], n_out[j], n_in, xq + off, xq2 + off, xd + off / 32, xs + off / 32, T,
                             yc[j], stream)))
                return st;
    }
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

int qmv_mv_multi_ep(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                    const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int ep_kind, int ep_j0,
                    int ep_j1, int* ep_counters, int8_t* ep_xq, int8_t* ep_xq2, float* ep_xd, float* ep_xs,
                    float* ep_a, void* stream) {
    if (!w || !n_out || !y || !ep_counters || !ep_xq || !ep_xq2 || !ep_xd || !ep_xs) return ST_NULL;
    if (n_jobs < 1 || n_jobs > kMaxJobs) return ST_BAD_TOKENS;
    if (ep_kind != 1 && ep_kind != 2) return ST_BAD_SHAPE;
    if (ep_j0 < 0 || ep_j0 >= n_jobs || (ep_kind == 2 && (ep_j1 < 0 || ep_j1 >= n_jobs || ep_j1 == ep_j0 || !ep_a)))
        return ep_kind == 2 && !ep_a ? ST_NULL : ST_BAD_SHAPE;
    if (n_out[ep_j0] % 32 || (ep_kind == 2 && n_out[ep_j1] != n_out[ep_j0])) return ST_BAD_SHAPE;
    if (!aligned(ep_counters, 4) || !aligned(ep_xq, 16) || !aligned(ep_xq2, 16) || !aligned(ep_xd, 4) ||
        !aligned(ep_xs, 4) || (ep_a && !aligned(ep_a, 4)))
        return ST_BAD_ALIGN;
    for (int j = 0; j < n_jobs; ++j) {
        const int st = check_mv(ggml_type, w[j], n_out[j], n_in, xq, xq2, xd, xs, y[j]);
        if (st) return st;
        if (!aligned(w[j], weight_align(ggml_type))) return ST_BAD_ALIGN;
    }
    const EpOut ep{ep_kind, ep_j0, ep_kind == 2 ? ep_j1 : -1, ep_counters, ep_xq, ep_xq2, ep_xd, ep_xs, ep_a};
    int st = ST_OK;
    if (tma_dense(ggml_type, n_jobs, w, n_out, y, n_in, xq, xq2, xd, xs, nullptr, 0, nullptr, nullptr,
                  static_cast<cudaStream_t>(stream), &st, nullptr, &ep))
        return st;
    return ST_BAD_SHAPE;        // the shape needs another kernel: qmv_mv_multi, then qmv_quant_q8 / qmv_act_q8
}

int qmv_mv_norm(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                const float* h, const float* r, float rs, float* h_out, const float* norm_w, float eps, void* stream) {
    if (!w || !n_out || !y || !h || !norm_w || (r && !h_out)) return ST_NULL;
    if (!known_format(ggml_type)) return ST_BAD_FORMAT;
    if (n_jobs < 1 || n_jobs > kMaxJobs) return ST_BAD_TOKENS;
    if (n_in <= 0 || n_in % block_values(ggml_type)) return ST_BAD_SHAPE;
    if (!aligned(h, 4) || !aligned(norm_w, 4) || (r && (!aligned(r, 4) || !aligned(h_out, 4)))) return ST_BAD_ALIGN;
    for (int j = 0; j < n_jobs; ++j) {
        if (!w[j] || !y[j]) return ST_NULL;
        if (n_out[j] <= 0) return ST_BAD_SHAPE;
        if (!aligned(w[j], weight_align(ggml_type)) || !aligned(y[j], 4)) return ST_BAD_ALIGN;
    }
    const NormIn norm{r, rs, h_out, norm_w, eps};
    int st = ST_OK;
    if (tma_dense(ggml_type, n_jobs, w, n_out, y, n_in, nullptr, nullptr, nullptr, nullptr, h, 1, nullptr, nullptr,
                  static_cast<cudaStream_t>(stream), &st, &norm))
        return st;
    return ST_BAD_SHAPE;        // the shape needs the fallback: qmv_norm_q8, then qmv_mv_multi
}

// workspace of qmv_moe_ffn: xq, xq2 (L dim bytes each), xd, xs (L dim / 32 floats each), aq, aq2, ad, as
// (the same for L k rows of ff), gs, us (L k rows of ff floats each), y (L k rows of dim floats), then
// the counters: one per (touched expert, 32-row group of ff), one per 4 rows of dim
namespace {
struct MoeWs {
    long long xq, xq2, xd, xs, aq, aq2, ad, as, gs, us, y, counters, n_gu, n_counters, total;
};
MoeWs moe_ws(int n_tok, int k, int dim, int ff, long long n_exp) {
    auto part = [](long long b) { return (b + 255) / 256 * 256; };
    const long long nx = (long long)n_tok * dim, na = (long long)n_tok * k * ff;
    MoeWs w{};
    long long o = 0;
    w.xq = o; o += part(nx);
    w.xq2 = o; o += part(nx);
    w.xd = o; o += part(nx / 8);
    w.xs = o; o += part(nx / 8);
    w.aq = o; o += part(na);
    w.aq2 = o; o += part(na);
    w.ad = o; o += part(na / 8);
    w.as = o; o += part(na / 8);
    w.gs = o; o += part(na * 4);
    w.us = o; o += part(na * 4);
    w.y = o; o += part((long long)n_tok * k * dim * 4);
    w.n_gu = std::min<long long>((long long)n_tok * k, n_exp) * (ff / 32);
    w.n_counters = w.n_gu + dim / kMoeRW;
    w.counters = o; o += part(w.n_counters * 4);
    w.total = o;
    return w;
}
}  // namespace

int64_t qmv_moe_workspace_bytes(int n_tok, int k, int dim, int ff) {
    if (n_tok <= 0 || k <= 0 || dim <= 0 || ff <= 0 || dim % 32 || ff % 32) return 0;
    return moe_ws(n_tok, k, dim, ff, kMoeMaxExperts).total;
}

int qmv_moe_ffn(int gate_up_type, const void* gate, const void* up, long long gate_up_per_expert, int down_type,
                const void* down, long long down_per_expert, long long n_exp, const long long* ids, const float* wts,
                int n_tok, int k, const void* x, int x_is_f32, long long x_stride, int dim, int ff, void* workspace,
                float* out, void* stream) {
    if (!known_format(gate_up_type) || !known_format(down_type)) return ST_BAD_FORMAT;
    if (!gate || !up || !down || !ids || !wts || !x || !workspace || !out) return ST_NULL;
    if (n_tok <= 0 || k <= 0 || (long long)n_tok * k > kMoeMaxPairs) return ST_BAD_TOKENS;
    if (n_exp <= 0 || n_exp > kMoeMaxExperts || dim <= 0 || ff <= 0 || x_stride < dim ||
        dim % block_values(gate_up_type) || ff % block_values(down_type) || dim % 32 || ff % 32)
        return ST_BAD_SHAPE;
    const long long gu_bytes = (long long)ff * (dim / block_values(gate_up_type)) * block_bytes(gate_up_type);
    const long long d_bytes = (long long)dim * (ff / block_values(down_type)) * block_bytes(down_type);
    if (gate_up_per_expert < gu_bytes || down_per_expert < d_bytes) return ST_BAD_SHAPE;
    if (!aligned(gate, weight_align(gate_up_type)) || !aligned(up, weight_align(gate_up_type)) ||
        !aligned(down, weight_align(down_type)) || gate_up_per_expert % weight_align(gate_up_type) ||
        down_per_expert % weight_align(down_type) || !aligned(workspace, 256) || !aligned(out, 4) ||
        !aligned(x, x_is_f32 ? 4 : 2))
        return ST_BAD_ALIGN;
    const long long nx = (long long)n_tok * dim;
    const MoeWs W = moe_ws(n_tok, k, dim, ff, n_exp);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    MoeParams P{};
    P.gate = static_cast<const uint8_t*>(gate);
    P.up = static_cast<const uint8_t*>(up);
    P.down = static_cast<const uint8_t*>(down);
    P.gate_per = P.up_per = gate_up_per_expert;
    P.down_per = down_per_expert;
    P.n_exp = n_exp;
    P.ids = ids;
    P.wts = wts;
    P.L = n_tok; P.k = k; P.dim = dim; P.ff = ff;
    int8_t* xq = reinterpret_cast<int8_t*>(ws + W.xq);
    int8_t* xq2 = reinterpret_cast<int8_t*>(ws + W.xq2);
    float* xd = reinterpret_cast<float*>(ws + W.xd);
    float* xs = reinterpret_cast<float*>(ws + W.xs);
    P.xq = xq; P.xq2 = xq2; P.xd = xd; P.xs = xs;
    P.aq = reinterpret_cast<int8_t*>(ws + W.aq);
    P.aq2 = reinterpret_cast<int8_t*>(ws + W.aq2);
    P.ad = reinterpret_cast<float*>(ws + W.ad);
    P.as = reinterpret_cast<float*>(ws + W.as);
    P.gs = reinterpret_cast<float*>(ws + W.gs);
    P.us = reinterpret_cast<float*>(ws + W.us);
    P.y = reinterpret_cast<float*>(ws + W.y);
    P.gu_done = reinterpret_cast<int*>(ws + W.counters);
    P.d_done = P.gu_done + W.n_gu;
    P.out = out;
    P.status = device_status_ptr();
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc = launch_pdl(moe_quant_kernel, dim3(unsigned((nx + 255) / 256)), dim3(256), st, x, x_is_f32, x_stride, dim,
                        nx, xq, xq2, xd, xs, P.gu_done, int(W.n_counters));
    if (rc) return rc;
    const long long touched = std::min<long long>((long long)n_tok * k, n_exp);
    const int grid_gu = int(std::min<long long>(touched * (ff / 32) * 16 / (kMoeThreads / 32) + 1, 1 << 20));
    rc = by_format(gate_up_type, [&](auto c) { return launch_moe_fmt<decltype(c)::value>(0, P, grid_gu, st); });
    if (rc) return rc;
    const int grid_d = int(std::min<long long>(touched * (dim / kMoeRW) / (kMoeThreads / 32) + 1, 1 << 20));
    return by_format(down_type, [&](auto c) { return launch_moe_fmt<decltype(c)::value>(1, P, grid_d, st); });
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
