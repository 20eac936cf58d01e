// Decode chain: a list of dependent single-token matvec stages in one persistent, cooperative launch.
//
// A stage is 1..4 matrices that read one input vector (q/k/v, o, gate/up, down).  Its input x is built
// from fp32 vectors by a fused producer (the reference runs these as separate kernels: norm_q8,
// akt_q8, the Eingang of mmvq.py:102-134, 825-849):
//   RAW       x = a
//   RMSNORM   v = a (+ b, written to h_out), x = v * rsqrt(mean(v^2) + eps) * norm_w
//   SILU_MUL  x = silu(a) * b  (b == null: silu(a))
// and quantised into the two-stage int8 activation (xq, xq2, xd, xs per 32 values) ONCE, in a global
// buffer of the workspace, 32 values (one group) per warp:
//   fed stage     the CTA that writes the last rows of a group of the previous stage's outputs (a
//                 counter per group in the workspace tells it) quantises that group right away;
//   other stages  the groups are split over the CTAs at the start of the stage, then a grid barrier.
// RMSNORM groups are quantised before the norm scale is known (u = v * norm_w, with the group's sum of
// v^2 stored beside it); the consumers multiply xd and xs by the scale when they load the activation.
// After a grid barrier every consumer lane loads its slice of the activation into registers and keeps
// it for the stage.  The producer warp never waits at these barriers: the weights do not depend on
// them, so it streams the next stages' tiles into the ring while the consumers wait.
//
// Two activation buffers alternate by stage parity: a buffer is rewritten only after a grid barrier
// that follows every CTA's last read of it.  Every spin (grid barrier, mbarrier) is bounded in time and
// sets a status bit on expiry.
#pragma once
#include "qmv_tma.cuh"

namespace qmv {

enum : int { CH_RAW = 0, CH_RMSNORM = 1, CH_SILU_MUL = 2 };
// consumer configurations compiled into the chain kernel (format, row length class)
enum : int { CFG_Q4K_4096 = 0, CFG_Q6K_14336 = 1, CFG_Q4K_14336 = 2, CFG_Q6K_4096 = 3, CFG_Q8_0_4096 = 4, CFG_COUNT = 5 };
constexpr int kChainMaxStages = 128;
constexpr int kChainNcw = 8;                        // consumer warps (measured: 8 beat 16, no spills)
constexpr int kChainMaxIn = 14336;                  // longest input vector a chain stage takes
constexpr int kChainMaxGroups = kChainMaxIn / 32;
constexpr int kChainPartFloats = 1024;              // deferred cross-warp partial sums (shared memory)
constexpr int kChainStageIn = 4096;                 // inputs up to this length are staged in shared memory
constexpr int kChainActSmem = 2 * kChainStageIn + 8 * (kChainStageIn / 32);
enum : int { DEV_BARRIER_TIMEOUT = 4 };

// workspace: [barrier counters 2 x kChainMaxStages][group counters 2 x kChainMaxGroups] (zeroed per
// launch), then two activation buffers [xq N][xq2 N][xd N/32][xs N/32][sum of squares N/32], N = kChainMaxIn
constexpr long long kChainCounterBytes = 4LL * (2 * kChainMaxStages + 2 * kChainMaxGroups);
constexpr long long kChainActBytes = 2LL * kChainMaxIn + 3LL * 4 * kChainMaxGroups;
constexpr long long kChainWorkspaceBytes = kChainCounterBytes + 2 * kChainActBytes;

struct ChainStage {
    const uint8_t* w[kMaxJobs];
    float* y[kMaxJobs];
    long long row_start[kMaxJobs + 1];
    const float* a;
    const float* b;
    const float* norm_w;
    float* h_out;
    long long row_bytes;
    long long total_rows;
    float eps;
    int n_out[kMaxJobs];
    int n_jobs, cfg, n_in, R, in_kind, wait;
    int fed;              // 1: the previous stage's CTAs quantise this stage's input as its groups complete
    int feed_mask;        // bit j: output of job j is an input vector of the NEXT stage (which is fed)
    int feed_target;      // rows of this stage that complete one group of the next stage's input
};

struct ChainParams {
    ChainStage st[kChainMaxStages];
    int n_stages;
    int S;                 // ring slots
    int F;                 // most copies in flight (1..S): the ring may hold more landed tiles than that
    int PF;                // tiles ahead of the copies that are prefetched into L2 (0: none)
    int slot_bytes;
    unsigned long long* trace;   // per (stage, CTA) timestamps (sweep builds; null otherwise)
    int* bar;              // grid-barrier counters: stage k done at [k], its input ready at [kChainMaxStages + k]
    int* cnt;              // group counters [buffer][group]
    int8_t* xq[2];
    int8_t* xq2[2];
    float* xd[2];
    float* xs[2];
    float* pss[2];         // per group: sum of v^2 (RMSNORM inputs)
    int* status;
};

// Base geometry of each configuration (for 16 consumer warps): team width G (lanes per row) and rows
// per tile R.  Tiles are 27..47 KB; 4 Q6_K rows give every CTA the same tile count for a 4096-row down
// projection.  Q6_K uses 32-value units here (F_Q6_K_U32): the 64-value units of the staged kernel need
// more registers than this non-inlined loop has.
__host__ __device__ constexpr int chain_cfg_g(int cfg) {
    return cfg == CFG_Q4K_4096 ? 64 : cfg == CFG_Q6K_14336 ? 512 : cfg == CFG_Q4K_14336 ? 256 : 128;
}
__host__ __device__ constexpr int chain_cfg_rows(int cfg) {
    return cfg == CFG_Q4K_4096 ? 16 : cfg == CFG_Q6K_14336 ? 4 : cfg == CFG_Q4K_14336 ? 4 : 8;
}
__host__ __device__ constexpr int chain_cfg_fmt(int cfg) {
    return cfg == CFG_Q4K_4096 || cfg == CFG_Q4K_14336 ? F_Q4_K : cfg == CFG_Q8_0_4096 ? F_Q8_0 : F_Q6_K;
}
__host__ __device__ constexpr int chain_cfg_nin(int cfg) {
    return cfg == CFG_Q6K_14336 || cfg == CFG_Q4K_14336 ? 14336 : 4096;
}
// The geometry for NCW consumer warps keeps each configuration's tile (R rows): with fewer warps a team
// is at most 32 NCW lanes wide (each lane then takes UPL units of its row) and takes more of the tile's
// rows (NPER), so every lane has more independent rows and units in flight.
template <int CFG, int NCW>
struct ChainCfg {
    static constexpr int FMT = chain_cfg_fmt(CFG) == F_Q6_K ? F_Q6_K_U32 : chain_cfg_fmt(CFG);
    static constexpr int G = chain_cfg_g(CFG) < 32 * NCW ? chain_cfg_g(CFG) : 32 * NCW;
    static constexpr int UPL = chain_cfg_g(CFG) / G;
    static constexpr int TEAMS = 32 * NCW / G;
    static constexpr int NPER = chain_cfg_rows(CFG) / TEAMS;
    static_assert(NPER * TEAMS == chain_cfg_rows(CFG), "tile rows split over the teams");
};
// the activation goes through shared memory when several teams would load the same units (every CTA
// reading the same few L2 lines many times over is slow); otherwise each lane loads its own units
template <int CFG, int NCW>
__host__ __device__ constexpr bool chain_cfg_staged() {
    return ChainCfg<CFG, NCW>::TEAMS > 1 && chain_cfg_nin(CFG) <= kChainStageIn;
}

// rows [c * total / grid, (c + 1) * total / grid) of a stage belong to CTA c
__device__ __forceinline__ int chain_row_begin(const ChainStage& st, int c) {
    return int((long long)c * st.total_rows / gridDim.x);
}

// A CTA's rows [lo, lo + n) of a stage's concatenated row space go in tiles of R rows from lo (the last
// one shorter).  A tile may span two jobs (one copy per job segment), so a CTA whose range crosses a
// job boundary runs no extra tile for it.
__device__ __forceinline__ int chain_job_of(const ChainStage& st, int g) {
    int j = 0;
    while (j + 1 < st.n_jobs && g >= int(st.row_start[j + 1])) ++j;
    return j;
}

// trace points of a sweep build: per (stage, CTA) kChainTraceFields words: four %globaltimer stamps, the
// ns thread 0 spent waiting for tile data in the stage, and the stage's tile count
enum : int { TR_ENTER = 0, TR_READY = 1, TR_DONE = 2, TR_FED = 3, TR_DATAWAIT = 4, TR_TILES = 5 };
constexpr int kChainTraceFields = 6;
__device__ __forceinline__ void chain_trace_set(const ChainParams& P, int k, int field, unsigned long long v) {
#ifdef QMV_TRACE
    if (P.trace && threadIdx.x == 0) P.trace[((long long)k * gridDim.x + blockIdx.x) * kChainTraceFields + field] = v;
#endif
}
__device__ __forceinline__ void chain_trace(const ChainParams& P, int k, int field) {
#ifdef QMV_TRACE
    chain_trace_set(P, k, field, global_ns());
#endif
}

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// grid barrier, arrive side: a release reduction by one thread after a CTA barrier makes the CTA's
// writes visible before the count
__device__ __forceinline__ void grid_arrive(int* counter) {
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.s32 [%0], 1;" :: "l"(counter) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}
// wait side: thread 0 spins (bounded) until every CTA has arrived, then all consumer threads go on
template <int NCW>
__device__ __forceinline__ void grid_wait(const int* counter, bool& dead, int* status) {
    if (threadIdx.x == 0 && !dead) {
        const unsigned long long t0 = global_ns();
        while (ld_acquire(counter) < int(gridDim.x)) {
            if (global_ns() - t0 > kWaitNs) {
                dead = true;
                if (status) atomicOr(status, DEV_BARRIER_TIMEOUT);
                break;
            }
        }
    }
    named_sync(kConsumerBarrier, 32 * NCW);
}

// ---- input production: one warp quantises group g (32 values) of stage `ns`'s input into buffer nb --

__device__ __forceinline__ void produce_group(const ChainParams& P, const ChainStage& ns, int nb, int g) {
    const int lane = threadIdx.x & 31;
    const int i = 32 * g + lane;
    float v = __ldcg(ns.a + i);
    if (ns.in_kind == CH_RMSNORM) {
        if (ns.b) {
            v += __ldcg(ns.b + i);
            if (ns.h_out) ns.h_out[i] = v;             // the residual stream after this add
        }
        const float ss = warp_sum(v * v);
        if (lane == 0) P.pss[nb][g] = ss;
        v *= __ldg(ns.norm_w + i);                   // the 1/rms factor is applied by the consumers
    } else if (ns.in_kind == CH_SILU_MUL) {
        v = v / (1.0f + expf(-v));
        if (ns.b) v *= __ldcg(ns.b + i);
    }
    quantize_group(v, i, P.xq[nb], P.xq2[nb], P.xd[nb], P.xs[nb]);
}

// ---- consumers of one stage ------------------------------------------------------------------------

// Not inlined: a kernel instance carries two configurations, and two inlined copies of this loop
// would share one register allocation and spill.  Returns the next ring iteration; *dead_io is the
// timed-out flag (read and written once per stage).
template <int CFG, int NCW>
__device__ __noinline__ int chain_consume(const ChainParams& P, const ChainStage& st, int k_stage, int it, int* dead_io,
                                          float* part, uint8_t* act_smem, uint32_t stage0, uint32_t full0,
                                          uint32_t empty0) {
    bool dead = *dead_io != 0;
    const int buf = k_stage & 1;
    using C = ChainCfg<CFG, NCW>;
    constexpr int FMT = C::FMT, G = C::G, UPL = C::UPL, NPER = C::NPER;
    constexpr int TEAMS = 32 * NCW / G;
    constexpr int WPT = G >= 32 ? G / 32 : 1;
    constexpr int VPU = UnitTraits<FMT>::VPU;
    constexpr int PR = kChainPartFloats / WPT;          // rows per window of deferred partial sums
    const int S = P.S;
    const uint32_t slot_bytes = uint32_t(P.slot_bytes);
    const int lane = threadIdx.x & 31;
    const int cl = threadIdx.x, team = cl / G, li = cl % G;
    const int U = st.n_in / VPU;
    // the 1/rms factor of an RMSNORM input: warp 0 issues the loads of the groups' sums of squares together
    // with the activation loads (one round trip for both) and adds them in a fixed order afterwards
    float* s_scale = reinterpret_cast<float*>(act_smem + kChainActSmem);
    float* s_pss = s_scale + 4;                          // kChainMaxGroups floats
    const bool rms = st.in_kind == CH_RMSNORM;
    auto pss_issue = [&]() {                             // asynchronous copies: no registers held
        if (threadIdx.x < 32 && rms) {
            for (int g = lane; g < st.n_in / 32; g += 32)
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" :: "r"(smem_u32(s_pss + g)), "l"(P.pss[buf] + g)
                             : "memory");
            asm volatile("cp.async.commit_group;" ::: "memory");
        }
    };
    auto norm_scale = [&]() {
        if (threadIdx.x < 32) {
            float scale = 1.f;
            if (rms) {
                asm volatile("cp.async.wait_all;" ::: "memory");
                __syncwarp();
                float ss = 0.f;
                for (int g = lane; g < st.n_in / 32; g += 32) ss += s_pss[g];
                scale = rsqrtf(warp_sum(ss) / float(st.n_in) + st.eps);
            }
            if (lane == 0) *s_scale = scale;
        }
    };
    Act<FMT> act[UPL];
    if constexpr (chain_cfg_staged<CFG, NCW>()) {
        int8_t* sq = reinterpret_cast<int8_t*>(act_smem);
        int8_t* sq2 = sq + kChainStageIn;
        float* sd = reinterpret_cast<float*>(sq2 + kChainStageIn);
        float* ss_ = sd + kChainStageIn / 32;
        const int n16 = st.n_in / 16, ng = st.n_in / 32;
        pss_issue();
        for (int i = cl; i < n16; i += 32 * NCW) {
            const int4 a = __ldcg(reinterpret_cast<const int4*>(P.xq[buf]) + i);
            const int4 b = __ldcg(reinterpret_cast<const int4*>(P.xq2[buf]) + i);
            const float d = i < ng ? __ldcg(P.xd[buf] + i) : 0.f;
            const float e = i < ng ? __ldcg(P.xs[buf] + i) : 0.f;
            reinterpret_cast<int4*>(sq)[i] = a;
            reinterpret_cast<int4*>(sq2)[i] = b;
            if (i < ng) {
                sd[i] = d;
                ss_[i] = e;
            }
        }
        norm_scale();
        named_sync(kConsumerBarrier, 32 * NCW);
#pragma unroll
        for (int i = 0; i < UPL; ++i) {
            const int u = li + G * i;
            if (u < U) load_act<FMT, true, SRC_SMEM>(act[i], u, sq, sq2, sd, ss_);
        }
    } else {
        pss_issue();
#pragma unroll
        for (int i = 0; i < UPL; ++i) {
            const int u = li + G * i;
            if (u < U) load_act<FMT, true, SRC_CG>(act[i], u, P.xq[buf], P.xq2[buf], P.xd[buf], P.xs[buf]);
        }
        norm_scale();
        named_sync(kConsumerBarrier, 32 * NCW);
    }
    if (st.in_kind == CH_RMSNORM) {
        const float scale = *s_scale;
#pragma unroll
        for (int i = 0; i < UPL; ++i) {
#pragma unroll
            for (int k = 0; k < UnitTraits<FMT>::NS; ++k) {
                act[i].d[k] *= scale;
                act[i].s[k] *= scale;
            }
        }
    }
    chain_trace(P, k_stage, TR_READY);
    int w_g0 = 0, w_rows = 0;                              // window: rows [w_g0, w_g0 + w_rows)
    auto flush = [&]() {                                    // every consumer thread, uniformly
        named_sync(kConsumerBarrier, 32 * NCW);
        if (!dead) {
            for (int rl = cl; rl < w_rows; rl += 32 * NCW) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < WPT; ++w) v += part[rl * WPT + w];
                const int g = w_g0 + rl, j = chain_job_of(st, g);
                st.y[j][g - int(st.row_start[j])] = v;
            }
        }
        named_sync(kConsumerBarrier, 32 * NCW);
        w_rows = 0;
    };
    const int lo = chain_row_begin(st, blockIdx.x), n = chain_row_begin(st, blockIdx.x + 1) - lo;
    const int R = st.R, tiles = (n + R - 1) / R;
    const uint32_t row_bytes = uint32_t(st.row_bytes);
#ifdef QMV_TRACE
    unsigned long long wait_ns = 0;
#endif
    for (int i = 0; i < tiles; ++i, ++it) {
        const int t0 = lo + i * R, nrows = min(R, n - i * R);
        const int s = it % S;
#ifdef QMV_TRACE
        const unsigned long long tw = threadIdx.x == 0 ? global_ns() : 0;
#endif
        const bool got = !dead && mbar_wait(full0 + 8 * s, (it / S) & 1);
#ifdef QMV_TRACE
        if (threadIdx.x == 0) wait_ns += global_ns() - tw;
#endif
        if (!got && !dead) {
            dead = true;
            if (lane == 0 && P.status) atomicOr(P.status, DEV_TIMEOUT);
        }
        const uint32_t stg = stage0 + uint32_t(s) * slot_bytes;
        float acc[NPER];
#pragma unroll
        for (int r = 0; r < NPER; ++r) acc[r] = 0.f;
        // every tile runs the full-tile code: rows past a short tile's end read stale bytes of the slot
        // (inside the slot, since R rows always fit) and their sums are never stored
        if (got) {
#pragma unroll
            for (int k = 0; k < UPL; ++k) {
                const int u = li + G * k;
                if (u < U) {
#pragma unroll
                    for (int r = 0; r < NPER; ++r)
                        acc[r] += unit_dot<FMT>(stg + uint32_t(team + TEAMS * r) * row_bytes, u, act[k], nullptr);
                }
            }
        }
        __syncwarp();
        if (got && lane == 0) mbar_arrive(empty0 + 8 * s);
        if constexpr (G <= 32) {
#pragma unroll
            for (int r = 0; r < NPER; ++r) {
                float v = acc[r];
#pragma unroll
                for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const int rr = team + TEAMS * r;
                if (li == 0 && got && rr < nrows) {
                    const int g = t0 + rr, j = chain_job_of(st, g);
                    st.y[j][g - int(st.row_start[j])] = v;
                }
            }
        } else {
            if (w_rows > 0 && (t0 != w_g0 + w_rows || w_rows + nrows > PR)) flush();
            if (w_rows == 0) w_g0 = t0;
            const int wt = li >> 5;
#pragma unroll
            for (int r = 0; r < NPER; ++r) {
                const float v = warp_sum(acc[r]);
                const int rr = team + TEAMS * r;
                if (lane == 0 && rr < nrows) part[(w_rows + rr) * WPT + wt] = v;
            }
            w_rows += nrows;
        }
    }
    if constexpr (G > 32) {
        if (w_rows > 0) flush();
    }
#ifdef QMV_TRACE
    chain_trace_set(P, k_stage, TR_DATAWAIT, wait_ns);
    chain_trace_set(P, k_stage, TR_TILES, (unsigned long long)tiles);
#endif
    *dead_io = dead;
    return it;
}

// ---- the producer's walk over every stage's tiles ---------------------------------------------------

// Position in the walk: stage k, tile i of this CTA's rows [lo, lo + n) of that stage.
struct ChainCursor {
    int k, i, lo, n;
};
__device__ __forceinline__ void chain_cursor_settle(const ChainParams& P, ChainCursor& c) {
    while (c.k < P.n_stages) {
        const ChainStage& st = P.st[c.k];
        c.lo = chain_row_begin(st, blockIdx.x);
        c.n = chain_row_begin(st, blockIdx.x + 1) - c.lo;
        if (c.i * st.R < c.n) return;
        ++c.k;
        c.i = 0;
    }
}
__device__ __forceinline__ void chain_cursor_next(const ChainParams& P, ChainCursor& c) {
    ++c.i;
    chain_cursor_settle(P, c);
}
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(p), "r"(bytes) : "memory");
}
// L2 prefetch of the tile at cursor c (every job segment; bulk sizes are multiples of 16 bytes)
__device__ __forceinline__ void chain_prefetch_tile(const ChainParams& P, const ChainCursor& c) {
    const ChainStage& st = P.st[c.k];
    const int t0 = c.lo + c.i * st.R, t1 = min(c.lo + c.n, t0 + st.R);
    for (int j = 0; j < st.n_jobs; ++j) {
        const int js = int(st.row_start[j]);
        const int a0 = max(t0, js), a1 = min(t1, int(st.row_start[j + 1]));
        if (a1 > a0) prefetch_l2(st.w[j] + (long long)(a0 - js) * st.row_bytes, uint32_t((a1 - a0) * st.row_bytes));
    }
}


// ---- the kernel ---------------------------------------------------------------------------------------
// shared memory: [S slots x slot_bytes][partial sums kChainPartFloats floats]
//                [staged activation kChainActSmem][scale 16 B][mbarriers 2 S]

__host__ __device__ constexpr int chain_red_bytes() { return kChainPartFloats * 4 + kChainActSmem + 16 + 4 * kChainMaxGroups; }

// CA, CB: the two consumer configurations this instance carries (a chain uses at most two; one
// kernel with all of them would spill registers)
template <int NCW, int CA, int CB>
__global__ void __launch_bounds__(32 * (NCW + 1), 1) chain_kernel(const __grid_constant__ ChainParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = P.S;
    float* part = reinterpret_cast<float*>(smem + (long long)S * P.slot_bytes);
    uint8_t* act_smem = smem + (long long)S * P.slot_bytes + kChainPartFloats * 4;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (long long)S * P.slot_bytes + chain_red_bytes());
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
    const uint32_t stage0 = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, NCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer: every stage's weight tiles, in order ----------------
        // At most F copies are in flight: a copy is issued once its slot is free AND the copy F tiles
        // back has landed.  The ring can then hold up to S landed tiles (while the consumers wait at a
        // stage boundary) without every slot's bytes queueing in the memory system at once, which
        // would delay the boundary's own small loads behind them.
        if (lane != 0) return;
        bool ok = true;
        ChainCursor c{0, 0, 0}, pf{0, 0, 0};
        chain_cursor_settle(P, c);
        chain_cursor_settle(P, pf);
        for (int a = 0; a < P.PF && pf.k < P.n_stages; ++a) {   // the prefetch cursor starts PF tiles ahead
            chain_prefetch_tile(P, pf);
            chain_cursor_next(P, pf);
        }
        int it = 0;
        for (; c.k < P.n_stages; ++it) {
            const int s = it % S;
            if (it >= S && !mbar_wait(empty0 + 8 * s, ((it / S) & 1) ^ 1)) {
                ok = false;
                break;
            }
            if (P.F < S && it >= P.F) {
                const int j = it - P.F;
                if (!mbar_wait(full0 + 8 * (j % S), (j / S) & 1)) {
                    ok = false;
                    break;
                }
            }
            const ChainStage& st = P.st[c.k];
            const int t0 = c.lo + c.i * st.R, t1 = min(c.lo + c.n, t0 + st.R);
            const long long row_bytes = st.row_bytes;
            mbar_arrive_tx(full0 + 8 * s, uint32_t((t1 - t0) * row_bytes));
            // one copy per job segment of the tile, into consecutive rows of the slot
            for (int j = 0; j < st.n_jobs; ++j) {
                const int js = int(st.row_start[j]);
                const int a0 = max(t0, js), a1 = min(t1, int(st.row_start[j + 1]));
                if (a1 <= a0) continue;
                bulk_g2s(stage0 + uint32_t(s) * uint32_t(P.slot_bytes) + uint32_t((a0 - t0) * row_bytes),
                         st.w[j] + (long long)(a0 - js) * row_bytes, uint32_t((a1 - a0) * row_bytes),
                         full0 + 8 * s);
            }
            chain_cursor_next(P, c);
            if (P.PF > 0 && pf.k < P.n_stages) {
                chain_prefetch_tile(P, pf);
                chain_cursor_next(P, pf);
            }
        }
        if (!ok) {
            if (P.status) atomicOr(P.status, DEV_TIMEOUT);
            for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(full0 + 8 * (k % S), (k / S) & 1);
        }
        return;
    }

    // ---------------- consumers ----------------
    int it = 0;
    bool dead = false;
    for (int k = 0; k < P.n_stages; ++k) {
        const ChainStage& st = P.st[k];
        const int buf = k & 1;
        chain_trace(P, k, TR_ENTER);
        if (st.wait && k > 0) grid_wait<NCW>(P.bar + (k - 1), dead, P.status);
        if (!st.fed) {
            // this stage quantises its own input: groups split over the CTAs, then a grid barrier
            const int ng = st.n_in / 32;
            const int g0 = int((long long)blockIdx.x * ng / gridDim.x), g1 = int((long long)(blockIdx.x + 1) * ng / gridDim.x);
            for (int g = g0 + warp; g < g1; g += NCW) produce_group(P, st, buf, g);
            named_sync(kConsumerBarrier, 32 * NCW);
            grid_arrive(P.bar + kChainMaxStages + k);
            grid_wait<NCW>(P.bar + kChainMaxStages + k, dead, P.status);
        }
        int dead_io = dead;
        if (st.cfg == CA)
            it = chain_consume<CA, NCW>(P, st, k, it, &dead_io, part, act_smem, stage0, full0, empty0);
        else
            it = chain_consume<CB, NCW>(P, st, k, it, &dead_io, part, act_smem, stage0, full0, empty0);
        dead = dead_io != 0;
        named_sync(kConsumerBarrier, 32 * NCW);            // this CTA's rows of stage k are written
        chain_trace(P, k, TR_DONE);
        if (k + 1 < P.n_stages && P.st[k + 1].fed) {
            // quantise every group of the next stage's input whose last rows this CTA wrote
            const ChainStage& ns = P.st[k + 1];
            const int nb = (k + 1) & 1;
            int* cnt = P.cnt + nb * kChainMaxGroups;
            const int lo = chain_row_begin(st, blockIdx.x), hi = chain_row_begin(st, blockIdx.x + 1);
            int p = 0;
            for (int j = 0; j < st.n_jobs; ++j) {
                if (!((st.feed_mask >> j) & 1)) continue;
                const int js = int(st.row_start[j]);
                const int a0 = max(lo, js) - js, a1 = min(hi, int(st.row_start[j + 1])) - js;
                if (a1 <= a0) continue;
                for (int g = a0 / 32; g <= (a1 - 1) / 32; ++g, ++p) {
                    if (p % NCW != warp) continue;
                    int last = 0;
                    if (lane == 0) {
                        const int mine = min(a1, 32 * g + 32) - max(a0, 32 * g);
                        const int old = atom_add_acq_rel(cnt + g, mine);   // releases this CTA's rows
                        last = old + mine == st.feed_target;
                        if (last) cnt[g] = 0;                // all contributions are in: ready for reuse
                    }
                    last = __shfl_sync(0xffffffffu, last, 0);
                    if (last && !dead) {
                        asm volatile("fence.acq_rel.gpu;" ::: "memory");
                        produce_group(P, ns, nb, g);
                    }
                }
            }
            named_sync(kConsumerBarrier, 32 * NCW);
        }
        chain_trace(P, k, TR_FED);
        grid_arrive(P.bar + k);
    }
}

}  // namespace qmv
