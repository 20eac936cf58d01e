// Decode chain: a list of dependent single-token matvec stages in one persistent, cooperative launch.
//
// A stage is 1..4 matrices that read one input vector (q/k/v, o, gate/up, down).  Its input is built
// inside the kernel by a fused producer from earlier outputs (the reference runs these as separate
// kernels: norm_q8, akt_q8, the Eingang of mmvq.py:102-134, 825-849):
//   RAW       x = a
//   RMSNORM   v = a (+ b, written to h_out), x = v * rsqrt(mean(v^2) + eps) * norm_w
//   SILU_MUL  x = silu(a) * b  (b == null: silu(a))
// and quantised into the two-stage int8 activation in shared memory.  Between a stage and the
// earlier stages it reads, the CTAs meet at a grid barrier (a counter per stage in the workspace,
// every spin bounded in time).  The producer warp never waits at these barriers: the weights do not
// depend on them, so it streams the next stages' tiles into the ring while the consumers wait.
#pragma once
#include "qmv_tma.cuh"

namespace qmv {

enum : int { CH_RAW = 0, CH_RMSNORM = 1, CH_SILU_MUL = 2 };
// consumer configurations compiled into the chain kernel (format, row length class)
enum : int { CFG_Q4K_4096 = 0, CFG_Q6K_14336 = 1, CFG_Q4K_14336 = 2, CFG_Q6K_4096 = 3, CFG_Q8_0_4096 = 4, CFG_COUNT = 5 };
constexpr int kChainMaxStages = 128;
constexpr int kChainNcw = 16;
enum : int { DEV_BARRIER_TIMEOUT = 4 };

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
};

struct ChainParams {
    ChainStage st[kChainMaxStages];
    int n_stages;
    int S;                 // ring slots
    int slot_bytes;
    int max_n_in;
    int* ws;               // one counter per stage (zeroed before the launch)
    int* status;
};

template <int CFG> struct ChainCfg;
template <> struct ChainCfg<CFG_Q4K_4096> { static constexpr int FMT = F_Q4_K, G = 64, UPL = 1, NPER = 2; };
template <> struct ChainCfg<CFG_Q6K_14336> { static constexpr int FMT = F_Q6_K, G = 256, UPL = 2, NPER = 2; };
template <> struct ChainCfg<CFG_Q4K_14336> { static constexpr int FMT = F_Q4_K, G = 256, UPL = 1, NPER = 2; };
template <> struct ChainCfg<CFG_Q6K_4096> { static constexpr int FMT = F_Q6_K, G = 128, UPL = 1, NPER = 2; };
template <> struct ChainCfg<CFG_Q8_0_4096> { static constexpr int FMT = F_Q8_0, G = 128, UPL = 1, NPER = 2; };

__host__ __device__ constexpr int chain_cfg_g(int cfg) {
    return cfg == CFG_Q4K_4096 ? 64 : cfg == CFG_Q6K_14336 ? 256 : cfg == CFG_Q4K_14336 ? 256 : 128;
}
__host__ __device__ constexpr int chain_cfg_nper(int cfg) { return 2; }
__host__ __device__ constexpr int chain_cfg_fmt(int cfg) {
    return cfg == CFG_Q4K_4096 || cfg == CFG_Q4K_14336 ? F_Q4_K : cfg == CFG_Q8_0_4096 ? F_Q8_0 : F_Q6_K;
}
__host__ __device__ constexpr int chain_cfg_nin(int cfg) {
    return cfg == CFG_Q6K_14336 || cfg == CFG_Q4K_14336 ? 14336 : 4096;
}

// rows [c * total / grid, (c + 1) * total / grid) of a stage belong to CTA c
__device__ __forceinline__ long long chain_row_begin(const ChainStage& st, int c) {
    return (long long)c * st.total_rows / gridDim.x;
}

__device__ __forceinline__ TileInfo chain_tile_at(const ChainStage& st, long long g, long long hi) {
    TileInfo t;
    int j = 0;
    while (j + 1 < st.n_jobs && g >= st.row_start[j + 1]) ++j;
    t.job = t.slot = j;
    t.row0 = int(g - st.row_start[j]);
    const long long lim = min(st.row_start[j + 1], hi);
    t.nrows = int(min((long long)st.R, lim - g));
    return t;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// ---- fused input producers (all consumer threads; x quantised into shared memory) ----------------

template <int NCW>
__device__ __forceinline__ float consumer_block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    named_sync(kConsumerBarrier, 32 * NCW);
    if (lane == 0) red[warp] = v;
    named_sync(kConsumerBarrier, 32 * NCW);
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) s += red[w];           // same order in every thread and every CTA
    return s;
}

// Each warp takes 32-value groups warp, warp + NCW, ... ; lane l holds value l of each.  Loads are
// issued CH groups at a time (independent loads, one L2 round trip per chunk) before any use.
template <int NCW>
__device__ void chain_input(const ChainStage& st, int8_t* xq, int8_t* xq2, float* xd, float* xs, float* red) {
    constexpr int CH = 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = st.n_in, ng = n / 32;
    const int mine = (ng - warp + NCW - 1) / NCW;             // groups of this warp
    const bool rms = st.in_kind == CH_RMSNORM, silu = st.in_kind == CH_SILU_MUL;
    const float* __restrict__ A = st.a;
    const float* __restrict__ B = st.b;
    float keep[CH];                                            // the values, when one chunk holds them all
    float scale = 1.f;
    if (rms) {
        float ss = 0.f;
        for (int c0 = 0; c0 < mine; c0 += CH) {
            float v[CH];
#pragma unroll
            for (int k = 0; k < CH; ++k) {
                const int i = 32 * (warp + NCW * (c0 + k)) + lane;
                v[k] = c0 + k < mine ? __ldcg(A + i) : 0.f;
            }
            if (B) {
#pragma unroll
                for (int k = 0; k < CH; ++k) {
                    const int i = 32 * (warp + NCW * (c0 + k)) + lane;
                    if (c0 + k < mine) v[k] += __ldcg(B + i);
                }
            }
#pragma unroll
            for (int k = 0; k < CH; ++k) {
                ss = fmaf(v[k], v[k], ss);
                keep[k] = v[k];
            }
        }
        scale = rsqrtf(consumer_block_sum<NCW>(ss, red) / float(n) + st.eps);
        if (st.h_out && B) {                          // the new residual stream: this CTA's share of it
            const long long lo = (long long)blockIdx.x * n / gridDim.x, hi = (long long)(blockIdx.x + 1) * n / gridDim.x;
            for (long long i = lo + threadIdx.x; i < hi; i += 32 * NCW) st.h_out[i] = __ldcg(A + i) + __ldcg(B + i);
        }
    }
    for (int c0 = 0; c0 < mine; c0 += CH) {
        float v[CH], w[CH];
        if (rms && mine <= CH) {
#pragma unroll
            for (int k = 0; k < CH; ++k) v[k] = keep[k];
        } else {
#pragma unroll
            for (int k = 0; k < CH; ++k) {
                const int i = 32 * (warp + NCW * (c0 + k)) + lane;
                v[k] = c0 + k < mine ? __ldcg(A + i) : 0.f;
            }
            if (B) {
#pragma unroll
                for (int k = 0; k < CH; ++k) {
                    const int i = 32 * (warp + NCW * (c0 + k)) + lane;
                    w[k] = c0 + k < mine ? __ldcg(B + i) : 0.f;
                }
#pragma unroll
                for (int k = 0; k < CH; ++k) v[k] = silu ? v[k] : v[k] + w[k];
            }
        }
        if (rms) {
#pragma unroll
            for (int k = 0; k < CH; ++k) {
                const int i = 32 * (warp + NCW * (c0 + k)) + lane;
                w[k] = c0 + k < mine ? __ldg(st.norm_w + i) : 0.f;
            }
        }
#pragma unroll
        for (int k = 0; k < CH; ++k) {
            if (c0 + k < mine) {                               // warp-uniform
                const int i = 32 * (warp + NCW * (c0 + k)) + lane;
                float x = v[k];
                if (rms) {
                    x = x * scale * w[k];
                } else if (silu) {
                    x = x / (1.0f + expf(-x));
                    if (B) x *= w[k];
                }
                quantize_group(x, i, xq, xq2, xd, xs);
            }
        }
    }
    named_sync(kConsumerBarrier, 32 * NCW);
}

// ---- consumers of one stage ------------------------------------------------------------------------

template <int CFG, int NCW>
__device__ void chain_consume(const ChainStage& st, int& it, bool& dead, const int8_t* sxq, const int8_t* sxq2,
                              const float* sxd, const float* sxs, float* red, uint32_t stage0, uint32_t slot_bytes,
                              int S, uint32_t full0, uint32_t empty0, int* status) {
    using C = ChainCfg<CFG>;
    constexpr int FMT = C::FMT, G = C::G, UPL = C::UPL, NPER = C::NPER;
    constexpr int TEAMS = 32 * NCW / G;
    constexpr int WPT = G >= 32 ? G / 32 : 1;
    constexpr int VPU = UnitTraits<FMT>::VPU;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cl = threadIdx.x, team = cl / G, li = cl % G;
    const int U = st.n_in / VPU;
    const uint2* grid = nullptr;
    Act<FMT> act[UPL];
#pragma unroll
    for (int i = 0; i < UPL; ++i) {
        const int u = li + G * i;
        if (u < U) load_act<FMT, true, false>(act[i], u, sxq, sxq2, sxd, sxs);
    }
    const long long hi = chain_row_begin(st, blockIdx.x + 1);
    for (long long g = chain_row_begin(st, blockIdx.x); g < hi; ++it) {
        const TileInfo ti = chain_tile_at(st, g, hi);
        g += ti.nrows;
        const int s = it % S;
        const bool got = !dead && mbar_wait(full0 + 8 * s, (it / S) & 1);
        if (!got && !dead) {
            dead = true;
            if (lane == 0 && status) atomicOr(status, DEV_TIMEOUT);
        }
        const uint32_t stg = stage0 + uint32_t(s) * slot_bytes;
        float acc[NPER];
#pragma unroll
        for (int i = 0; i < NPER; ++i) acc[i] = 0.f;
        if (got && ti.nrows == NPER * TEAMS && st.R == NPER * TEAMS) {
#pragma unroll
            for (int k = 0; k < UPL; ++k) {
                const int u = li + G * k;
                if (u < U) {
#pragma unroll
                    for (int i = 0; i < NPER; ++i)
                        acc[i] += unit_dot<FMT>(stg + uint32_t((team + TEAMS * i) * st.row_bytes), u, act[k], grid);
                }
            }
        } else if (got) {
#pragma unroll
            for (int i = 0; i < NPER; ++i) {
                const int r = team + TEAMS * i;
                if (r < ti.nrows) {
#pragma unroll
                    for (int k = 0; k < UPL; ++k) {
                        const int u = li + G * k;
                        if (u < U) acc[i] += unit_dot<FMT>(stg + uint32_t(r * st.row_bytes), u, act[k], grid);
                    }
                }
            }
        }
        __syncwarp();
        if (got && lane == 0) mbar_arrive(empty0 + 8 * s);
        float* y = st.y[ti.job];
        if constexpr (G <= 32) {
#pragma unroll
            for (int i = 0; i < NPER; ++i) {
                float v = acc[i];
#pragma unroll
                for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                const int r = team + TEAMS * i;
                if (li == 0 && got && r < ti.nrows) y[ti.row0 + r] = v;
            }
        } else {
            float* rb = red + (it & 1) * NCW * NPER;
#pragma unroll
            for (int i = 0; i < NPER; ++i) {
                const float v = warp_sum(acc[i]);
                if (lane == 0) rb[warp * NPER + i] = v;
            }
            named_sync(1 + team, G);
            const int wt = li >> 5;
            if (got && wt == 0 && lane < NPER) {
                const int r = team + TEAMS * lane;
                if (r < ti.nrows) {
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < WPT; ++w) v += rb[(team * WPT + w) * NPER + lane];
                    y[ti.row0 + r] = v;
                }
            }
        }
    }
}

// ---- the kernel ---------------------------------------------------------------------------------------
// shared memory: [S slots x slot_bytes][reduction 2 x NCW x 4 floats][block-sum 32 floats]
//                [activation xq K, xq2 K, xd K/32, xs K/32 (K = max n_in)][mbarriers]

__host__ __device__ constexpr int chain_red_bytes(int ncw) { return 2 * ncw * 4 * 4 + 32 * 4; }

// CA, CB: the two consumer configurations this instance carries (a chain uses at most two; one
// kernel with all of them would spill registers)
template <int NCW, int CA, int CB>
__global__ void __launch_bounds__(32 * (NCW + 1), 1) chain_kernel(const __grid_constant__ ChainParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = P.S;
    uint8_t* red_p = smem + (long long)S * P.slot_bytes;
    float* red = reinterpret_cast<float*>(red_p);
    float* bsum = red + 2 * NCW * 4;
    uint8_t* act_p = red_p + chain_red_bytes(NCW);
    int8_t* sxq = reinterpret_cast<int8_t*>(act_p);
    int8_t* sxq2 = sxq + P.max_n_in;
    float* sxd = reinterpret_cast<float*>(sxq2 + P.max_n_in);
    float* sxs = sxd + P.max_n_in / 32;
    uint64_t* bars = reinterpret_cast<uint64_t*>(act_p + tma_act_bytes(P.max_n_in));
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
        if (lane != 0) return;
        int it = 0;
        bool ok = true;
        for (int k = 0; k < P.n_stages && ok; ++k) {
            const ChainStage& st = P.st[k];
            const long long hi = chain_row_begin(st, blockIdx.x + 1);
            for (long long g = chain_row_begin(st, blockIdx.x); g < hi; ++it) {
                const int s = it % S;
                if (it >= S && !mbar_wait(empty0 + 8 * s, ((it / S) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                const TileInfo ti = chain_tile_at(st, g, hi);
                g += ti.nrows;
                const uint32_t bytes = uint32_t((long long)ti.nrows * st.row_bytes);
                mbar_arrive_tx(full0 + 8 * s, bytes);
                bulk_g2s(stage0 + uint32_t(s) * uint32_t(P.slot_bytes), st.w[ti.job] + (long long)ti.row0 * st.row_bytes,
                         bytes, full0 + 8 * s);
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
        if (st.wait && k > 0) {
            // grid barrier: every CTA has written its rows of stage k-1 (and so of all earlier stages)
            if (threadIdx.x == 0 && !dead) {
                const unsigned long long t0 = global_ns();
                while (ld_acquire(P.ws + (k - 1)) < int(gridDim.x)) {
                    if (global_ns() - t0 > kWaitNs) {
                        dead = true;
                        if (P.status) atomicOr(P.status, DEV_BARRIER_TIMEOUT);
                        break;
                    }
                }
            }
            named_sync(kConsumerBarrier, 32 * NCW);
        }
        chain_input<NCW>(st, sxq, sxq2, sxd, sxs, bsum);
        if (st.cfg == CA)
            chain_consume<CA, NCW>(st, it, dead, sxq, sxq2, sxd, sxs, red, stage0, P.slot_bytes, S, full0, empty0, P.status);
        else
            chain_consume<CB, NCW>(st, it, dead, sxq, sxq2, sxd, sxs, red, stage0, P.slot_bytes, S, full0, empty0, P.status);
        // this CTA's rows of stage k are written: count it (the stores are ordered before the release)
        named_sync(kConsumerBarrier, 32 * NCW);
        if (threadIdx.x == 0) {
            __threadfence();
            atomicAdd(P.ws + k, 1);
        }
    }
}

}  // namespace qmv
