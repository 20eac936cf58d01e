// Host side of the tensor-core tile path (qmv_tc.cuh): planning, workspace layout, launches, C ABI.
#include <algorithm>

#include "qmv_host.cuh"
#include "qmv_tc.cuh"
#include "../../include/nemicli_qmv.h"

using namespace qmv;

namespace {

bool tc_format(int f) { return f == F_Q4_K || f == F_Q6_K; }

// resident CTAs per SM at this shared-memory size: by shared memory (233472 B an SM, 1 KB reserved per
// CTA beside its static 1 KB) and by registers (the kernel's count, read once; 168 if unavailable).  No
// runtime occupancy query: the plan must come out the same for the workspace size and the launch.
template <int FMT>
int tc_occupancy(int n_pad) {
    static int regs = 0;
    if (regs == 0) {
        cudaFuncAttributes fa{};
        regs = cudaFuncGetAttributes(&fa, tc_mm_kernel<FMT>) == cudaSuccess && fa.numRegs > 0 ? fa.numRegs : 168;
    }
    const int by_smem = 233472 / (tc_smem(n_pad) + 2048);
    const int per_warp = (regs * 32 + 255) / 256 * 256;
    const int by_regs = 65536 / (per_warp * (kTcThreads / 32));
    return std::max(1, std::min({by_smem, by_regs, 32}));
}

// row tiles x K parts: at most one wave of resident CTAs, each part at least four K steps so that its
// stages overlap, and the parts' sums (n_tok x n_out fp32 each) not more bytes than the weights.  Planned
// for the first group of tokens (the largest) and kept for every group.
struct TcPlan {
    int tiles, splits, chunks, n_pad;
};
TcPlan tc_plan(int fmt, int n_out, int n_in, int n_tok) {
    TcPlan p{};
    const int g = std::min(n_tok, kTcMaxN);
    p.n_pad = (g + 15) / 16 * 16;
    p.tiles = (n_out + kTcRows - 1) / kTcRows;
    p.chunks = n_in / kTcK;
    const int occ = fmt == F_Q4_K ? tc_occupancy<F_Q4_K>(p.n_pad) : tc_occupancy<F_Q6_K>(p.n_pad);
    const int wave = std::max(1, occ * sm_count() / p.tiles);
    const long long wbytes = (long long)n_out * (n_in / 256) * block_bytes(fmt);
    const long long pbytes = (long long)g * n_out * 4;
    const int traffic = int(std::max<long long>(1, wbytes / std::max<long long>(1, pbytes)));
    p.splits = std::max(1, std::min({wave, p.chunks / 4, traffic, 32}));
    return p;
}

struct TcWs {
    long long xh, xs, part, done, total;
};
TcWs tc_ws(int fmt, int n_out, int n_in, int n_tok) {
    auto part = [](long long b) { return (b + 255) / 256 * 256; };
    const TcPlan pl = tc_plan(fmt, n_out, n_in, n_tok);
    const long long g = std::min(n_tok, kTcMaxN);
    TcWs w{};
    long long o = 0;
    w.xh = o; o += part(g * n_in * 2);
    w.xs = o; o += part(g * 4);
    w.part = o; o += pl.splits > 1 ? part((long long)pl.splits * g * n_out * 4) : 0;
    w.done = o; o += part((long long)pl.tiles * 4);
    w.total = o;
    return w;
}

template <int FMT>
int launch_tc(const TcParams& P, int grid, cudaStream_t st) {
    static bool attr = false;                        // more than 48 KB of dynamic shared memory
    if (!attr) {
        if (cudaFuncSetAttribute(tc_mm_kernel<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem) != cudaSuccess)
            return launched();
        attr = true;
    }
    tc_mm_kernel<FMT><<<grid, kTcThreads, tc_smem(P.n_pad), st>>>(P);
    return launched();
}

}  // namespace

extern "C" {

int64_t qmv_mm_tc_workspace_bytes(int ggml_type, int n_out, int n_in, int n_tok) {
    if (!tc_format(ggml_type) || n_out <= 0 || n_in <= 0 || n_in % 256 || n_tok <= 0) return 0;
    return tc_ws(ggml_type, n_out, n_in, n_tok).total;
}

int qmv_mm_tc(int ggml_type, const uint8_t* w, int n_out, int n_in, const void* x, int x_is_f32, int n_tok,
              float* y, void* workspace, long long workspace_bytes, void* stream) {
    if (!tc_format(ggml_type)) return ST_BAD_FORMAT;
    if (!w || !x || !y || !workspace) return ST_NULL;
    if (n_out <= 0 || n_in <= 0 || n_in % 256) return ST_BAD_SHAPE;
    if (n_tok <= 0) return ST_BAD_TOKENS;
    if (!aligned(w, ggml_type == F_Q4_K ? 16 : 2) || !aligned(x, x_is_f32 ? 4 : 2) || !aligned(y, 4) ||
        !aligned(workspace, 256))
        return ST_BAD_ALIGN;
    const long long row_bytes = (long long)(n_in / 256) * block_bytes(ggml_type);
    const TcPlan pl = tc_plan(ggml_type, n_out, n_in, n_tok);
    const TcWs W = tc_ws(ggml_type, n_out, n_in, n_tok);
    if (workspace_bytes < W.total) return ST_BAD_SHAPE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int t0 = 0; t0 < n_tok; t0 += kTcMaxN) {          // groups of at most 128 tokens
        const int g = std::min(kTcMaxN, n_tok - t0);
        TcParams P{};
        P.w = w;
        P.row_bytes = row_bytes;
        P.n_out = n_out;
        P.n_in = n_in;
        P.xh = reinterpret_cast<const uint16_t*>(ws + W.xh);
        P.xs = reinterpret_cast<const float*>(ws + W.xs);
        P.n_tok = g;
        P.n_pad = (g + 15) / 16 * 16;
        P.splits = pl.splits;
        P.part = reinterpret_cast<float*>(ws + W.part);
        P.done = reinterpret_cast<int*>(ws + W.done);
        P.y = y + (long long)t0 * n_out;
        P.status = device_status_ptr();
        const uint8_t* xg = static_cast<const uint8_t*>(x) + (long long)t0 * n_in * (x_is_f32 ? 4 : 2);
        tc_input_kernel<<<g, 256, 0, st>>>(xg, x_is_f32, n_in, reinterpret_cast<uint16_t*>(ws + W.xh),
                                           reinterpret_cast<float*>(ws + W.xs), P.done, pl.tiles);
        int rc = launched();
        if (rc) return rc;
        const int grid = pl.tiles * pl.splits;
        rc = ggml_type == F_Q4_K ? launch_tc<F_Q4_K>(P, grid, st) : launch_tc<F_Q6_K>(P, grid, st);
        if (rc) return rc;
    }
    return ST_OK;
}

}  // extern "C"
