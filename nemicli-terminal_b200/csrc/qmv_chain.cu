// Decode chain: host side of chain_kernel (qmv_chain.cuh) and the C-ABI entry points qmv_chain,
// qmv_chain_noalloc and qmv_chain_workspace_bytes (declarations: include/nemicli_qmv.h).
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include <cuda.h>

#include "qmv_host.cuh"
#include "qmv_chain.cuh"
#include "../../include/nemicli_qmv.h"

using namespace qmv;

namespace {

// Workspace of qmv_chain_noalloc (barrier and group counters, activation buffers), for callers that
// cannot allocate.
static __device__ __align__(256) uint8_t g_chain_workspace[QMV_CHAIN_WORKSPACE_BYTES];
static_assert(QMV_CHAIN_NOALLOC_MAX_STAGES <= kChainMaxStages, "more stages than a chain takes");
static_assert(QMV_CHAIN_WORKSPACE_BYTES == kChainWorkspaceBytes, "workspace size in the header is stale");

// Address of g_chain_workspace in the current context of the current device.  The address is looked
// up once per context (with that context current) and cached together with the context's unique id, so
// a context torn down and created again (cudaDeviceReset, a primary context released by every user) gets
// a fresh lookup instead of a stale pointer.  Null if the lookup fails (its cudaError_t goes to
// qmv_last_cuda_error).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

bool current_context_id(unsigned long long* id) {
    static CtxGetCurrentFn get_current = nullptr;
    static CtxGetIdFn get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<CtxGetCurrentFn>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<CtxGetIdFn>(f);
        cudaGetLastError();
    });
    if (!get_current || !get_id) return false;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return false;
    return get_id(ctx, id) == CUDA_SUCCESS;
}

void* chain_workspace_ptr() {
    static std::mutex mu;
    static void* cache[64] = {nullptr};
    static unsigned long long cache_ctx[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    unsigned long long ctx = 0;
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev] && current_context_id(&ctx) && cache_ctx[dev] == ctx) return cache[dev];
    // first call in this context (the lookup makes the device's primary context current if no context is)
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_chain_workspace);
    if (e != cudaSuccess || !p) {
        set_last_cuda_error(int(e != cudaSuccess ? e : cudaErrorInvalidSymbol));
        cudaGetLastError();                    // do not leave the error for the next launch check
        cache[dev] = nullptr;
        return nullptr;
    }
    cache[dev] = p;
    cache_ctx[dev] = current_context_id(&ctx) ? ctx : 0;   // 0: no id, so every call looks it up again
    return p;
}

// Ring of the decode chain: slots, most copies in flight, tiles prefetched into L2 ahead of the copies.
// Fixed in the shipped library; a -DQMV_SWEEP build reads NEMICLI_CHAIN_SLOTS / _INFLIGHT / _PF.
struct ChainRing {
    int slots = 3, inflight = 0, prefetch = 0, ncw = kChainNcw;
    ChainRing() {
#ifdef QMV_SWEEP
        if (const char* e = std::getenv("NEMICLI_CHAIN_NCW")) ncw = std::atoi(e) == 16 ? 16 : 8;
        if (const char* e = std::getenv("NEMICLI_CHAIN_SLOTS")) slots = std::atoi(e);
        if (const char* e = std::getenv("NEMICLI_CHAIN_INFLIGHT")) inflight = std::atoi(e);
        if (const char* e = std::getenv("NEMICLI_CHAIN_PF")) prefetch = std::atoi(e);
#endif
    }
};
const ChainRing& chain_ring() {
    static const ChainRing r;
    return r;
}
unsigned long long* g_chain_trace = nullptr;

// the kernel instance for NCW consumer warps and a pair of configurations (a chain uses at most two)
template <int NCW>
void (*chain_kernel_pair(int pair))(const ChainParams) {
    return pair == 0 ? chain_kernel<NCW, CFG_Q4K_4096, CFG_Q6K_14336>
         : pair == 1 ? chain_kernel<NCW, CFG_Q4K_4096, CFG_Q4K_14336>
         : pair == 2 ? chain_kernel<NCW, CFG_Q6K_4096, CFG_Q6K_14336>
                     : chain_kernel<NCW, CFG_Q8_0_4096, CFG_Q6K_4096>;
}
void (*chain_kernel_for(int ncw, int pair))(const ChainParams) {
#ifdef QMV_SWEEP
    if (ncw == 16) return chain_kernel_pair<16>(pair);
#endif
    return ncw == kChainNcw ? chain_kernel_pair<kChainNcw>(pair) : nullptr;
}   // per (stage, CTA) timestamps: sweep builds only

}  // namespace

extern "C" {

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
        c.R = chain_cfg_rows(cfg);
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
    const ChainRing ring = chain_ring();
    if (ring.slots >= 2 && ring.slots < S) S = ring.slots;
    if (S > 32) S = 32;
    if (S < 2) return ST_BAD_SHAPE;
    P.F = ring.inflight >= 1 && ring.inflight < S ? ring.inflight : int(S);
    P.PF = ring.prefetch;
    P.trace = g_chain_trace;
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
    const int ncw = ring.ncw;
    void (*kern)(const ChainParams) = chain_kernel_for(ncw, pair);
    if (!kern) return ST_BAD_SHAPE;
    static int configured[64][2][4] = {{{0}}};
    const int wi = ncw == kChainNcw ? 0 : 1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev][wi][pair]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess)
            return launched();
        configured[dev][wi][pair] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count());
    cfg.blockDim = dim3(32 * (ncw + 1));
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
    if (!ws) return ST_LAUNCH;                                // the cudaError_t is in qmv_last_cuda_error
    return qmv_chain(stages, n_stages, ws, stream);           // clears the counters on `stream`
}

#ifdef QMV_TRACE
// sweep builds: device buffer of n_stages x grid x 4 uint64 stamps for the next chain launches (null: off)
int qmv_chain_set_trace(void* buf) {
    g_chain_trace = static_cast<unsigned long long*>(buf);
    return ST_OK;
}
#endif

}  // extern "C"
