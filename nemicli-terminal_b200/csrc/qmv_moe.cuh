// Grouped mixture-of-experts FFN driven by router ids on the device (the reference's expert path:
// models/moe.py:264-321 over PackedExperts, models/common.py:462-475, cudakern.py:756-774):
//
//     out[t] = sum_j w[t, j] * down_e(silu(gate_e x_t) * up_e x_t),   e = ids[t, j]
//
// in three kernels, the two matrix ones each reading every expert the call touches once, whatever
// number of tokens chose it:
//
//   moe_quant_kernel   the token rows (row stride x_stride values) into the activation input, and the
//                      two kernels' counters to zero;
//   moe_gateup_kernel  warp unit = (touched expert, 32-row group g, quad q of kMoeRW rows among that
//                      group's 32 gate rows and 32 up rows): the rows are multiplied with the inputs of
//                      the expert's pairs, kMoeChunk pairs at a time, into gate / up sums (workspace).
//                      The last of a group's quads to finish (a counter per (expert, group)) forms silu(g) * u of
//                      the group's 32 values for each pair and quantises them into that pair's down
//                      input;
//   moe_down_kernel    warp unit = (touched expert, kMoeRW rows of down): the rows times the expert's
//                      pairs' inputs into y (one row of dim per pair, workspace).  The last expert to
//                      finish a block of rows (a counter per block) takes each token's sum over its slots for
//                      those rows, in slot order (deterministic, the order of the reference's weighted
//                      sum).
//
// Units are independent (no block barrier after the grouping): each warp walks its units with an L2
// prefetch of the next one's weight rows (contiguous per expert) issued before the current one.
//
// Every CTA of the two matrix kernels derives the grouping itself from ids (at most kMoeMaxPairs pairs,
// n_exp at most kMoeMaxExperts): a counting sort of the valid pairs by expert, stable in the pair index,
// and the touched experts ascending.  Ids outside [0, n_exp) add nothing (a -1 marks an unused slot;
// any other such id also sets QMV_DEV_BAD_ADDRESS).  Weight rows go through the per-format lanes of the
// warp-per-row kernel (qmv_kernels.cuh).
#pragma once
#include <type_traits>

#include "qmv_kernels.cuh"

namespace qmv {

constexpr int kMoeMaxPairs = 1024;     // tokens x slots of one call
constexpr int kMoeMaxExperts = 1024;   // experts addressable by one call
#if defined(QMV_SWEEP) && defined(QMV_MOE_RW)
constexpr int kMoeRW = QMV_MOE_RW, kMoeChunk = QMV_MOE_CHUNK, kMoeThreads = QMV_MOE_THREADS,
              kMoeMinBlocks = QMV_MOE_MINB;
#else
constexpr int kMoeRW = 4;              // rows per warp unit
constexpr int kMoeChunk = 4;           // pairs multiplied per pass over a weight row
constexpr int kMoeThreads = 512;       // 16 warps a CTA
constexpr int kMoeMinBlocks = 1;       // resident CTAs per SM the register budget is set for
#endif
constexpr int kMoeQuads = 64 / kMoeRW; // units of one (expert, 32-row group): its 32 gate and 32 up rows

struct MoeParams {
    const uint8_t* gate;
    const uint8_t* up;
    const uint8_t* down;
    long long gate_per, up_per, down_per;   // bytes per expert
    long long n_exp;
    const long long* ids;                   // (L, k)
    const float* wts;                       // (L, k)
    int L, k, dim, ff;
    const int8_t* xq;                       // quantised x: L rows of dim
    const int8_t* xq2;
    const float* xd;
    const float* xs;
    int8_t* aq;                             // down inputs: L * k rows of ff (one per pair)
    int8_t* aq2;
    float* ad;
    float* as;
    float* gs;                              // gate sums: L * k rows of ff
    float* us;                              // up sums: L * k rows of ff
    float* y;                               // down results: L * k rows of dim
    int* gu_done;                           // per (touched expert, group): quads finished
    int* d_done;                            // per 4-row block of dim: experts finished
    float* out;                             // (L, dim)
    int* status;
};

// the call's grouping, built by every CTA in shared memory
struct MoeRoute {
    int nu;                             // touched experts
    int nv;                             // valid pairs
    short expert[kMoeMaxPairs];         // ascending
    short start[kMoeMaxPairs + 1];      // their pairs: pair[start[u] .. start[u + 1])
    short pair[kMoeMaxPairs];           // p = t * k + j, ascending within an expert
    int cur[kMoeMaxExperts];            // per expert: pair count, then the next free position
    short ex[kMoeMaxPairs];             // per pair: its expert, -1 if it is not valid
};

__device__ __forceinline__ int lane_mask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return int(m);
}

// All threads of the block: counting sort of the valid pairs by expert.  A histogram with shared
// atomics; then warp 0 scans the counts, lists the touched experts and places the pairs in index
// order, 32 at a time, the lanes of one expert ranked by __match_any_sync, so that the order within an
// expert is the pair order.
__device__ __forceinline__ void moe_route(const MoeParams& P, MoeRoute& R) {
    const int n = P.L * P.k, ne = int(P.n_exp);
    for (int e = threadIdx.x; e < ne; e += blockDim.x) R.cur[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < n; p += blockDim.x) {
        const long long e = P.ids[p];
        const bool ok = e >= 0 && e < P.n_exp;
        if (!ok && e != kPadSlot && P.status) atomicOr(P.status, DEV_BAD_ADDRESS);
        R.ex[p] = ok ? short(e) : short(-1);
        if (ok) atomicAdd(&R.cur[e], 1);
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int lane = threadIdx.x;
        int base = 0, nu = 0;
        for (int e0 = 0; e0 < ne; e0 += 32) {
            const int e = e0 + lane;
            const int c = e < ne ? R.cur[e] : 0;
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const unsigned used = __ballot_sync(0xffffffffu, c > 0);
            if (c > 0) {
                const int u = nu + __popc(used & unsigned(lane_mask_lt()));
                R.expert[u] = short(e);
                R.start[u] = short(base + incl - c);
            }
            if (e < ne) R.cur[e] = base + incl - c;
            base += __shfl_sync(0xffffffffu, incl, 31);
            nu += __popc(used);
        }
        if (lane == 0) {
            R.nu = nu;
            R.nv = base;
            R.start[nu] = short(base);
        }
        __syncwarp();
        for (int p0 = 0; p0 < n; p0 += 32) {
            const int p = p0 + lane;
            const int e = p < n ? R.ex[p] : -1;
            const unsigned same = __match_any_sync(0xffffffffu, e);
            int pos = 0;
            if (e >= 0) pos = R.cur[e] + __popc(same & unsigned(lane_mask_lt()));
            __syncwarp();
            if (e >= 0) {
                R.pair[pos] = short(p);
                if ((same & unsigned(lane_mask_lt())) == 0) R.cur[e] += __popc(same);   // lowest lane of the expert
            }
            __syncwarp();
        }
    }
    __syncthreads();
}

// token rows of dim values, x_stride values apart -> the activation input (L rows of dim, dense)
static __global__ void __launch_bounds__(256) moe_quant_kernel(const void* __restrict__ x, int x_f32, long long x_stride,
                                                        int dim, long long n, int8_t* __restrict__ xq,
                                                        int8_t* __restrict__ xq2, float* __restrict__ xd,
                                                        float* __restrict__ xs, int* __restrict__ counters,
                                                        int n_counters) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");           // nothing touched before the previous kernel ends
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (long long c = i; c < n_counters; c += (long long)gridDim.x * blockDim.x) counters[c] = 0;
    if ((i & ~31LL) >= n) return;          // dim % 32 == 0: whole warps leave together
    const long long src = (i / dim) * x_stride + i % dim;
    const float v = x_f32 ? static_cast<const float*>(x)[src] : bf2f(static_cast<const uint16_t*>(x)[src]);
    quantize_group(v, i, xq, xq2, xd, xs);
}

// f(std::integral_constant<int, T>) for T = n, 1 <= n <= kMoeChunk
template <int T = 1, class F>
__device__ __forceinline__ void moe_with_t(int n, F&& f) {
    if constexpr (T < kMoeChunk) {
        if (n != T) return moe_with_t<T + 1>(n, f);
    }
    f(std::integral_constant<int, T>{});
}

// RW consecutive rows starting at `row0` of one expert matrix (n_in values a row, rows of row_bytes)
// against T inputs whose value offsets are tk.tb (activation pointers in A), one warp; every lane gets
// the sums.
template <int FMT, int T, int RW>
__device__ __forceinline__ void moe_rows(const uint8_t* base, long long row_bytes, int row0, int n_in,
                                         const MvParams& A, const Tok<T>& tk, float (&acc)[RW][T],
                                         const uint2* grid) {
    const int lane = threadIdx.x & 31, q = lane & 7, sb0 = lane >> 3;
    const uint8_t* rows[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) rows[r] = base + (long long)(row0 + r) * row_bytes;
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int t = 0; t < T; ++t) acc[r][t] = 0.f;
    const int n_sb = (n_in + 255) >> 8;
    for (int sb = sb0; sb < n_sb; sb += 4) lane_any<FMT, T, RW, false>(rows, sb, q, A, tk, acc, row0, grid);
#pragma unroll
    for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int t = 0; t < T; ++t) acc[r][t] = warp_sum(acc[r][t]);
}

// L2 prefetch of [p, p + bytes) by one lane, trimmed inward to 16-byte boundaries (bulk granularity)
__device__ __forceinline__ void moe_prefetch(const uint8_t* p, long long bytes) {
    const uintptr_t a0 = (reinterpret_cast<uintptr_t>(p) + 15) & ~uintptr_t(15);
    const uintptr_t a1 = (reinterpret_cast<uintptr_t>(p) + uintptr_t(bytes)) & ~uintptr_t(15);
    if (a1 > a0)
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(a0), "r"(uint32_t(a1 - a0)) : "memory");
}

// T pairs' sums of RW rows -> dst[pair][row0 .. row0 + RW) (rows n_cols apart), lane t stores pair t
template <int T, int RW>
__device__ __forceinline__ void moe_store(float* dst, int n_cols, int row0, const short* pr, const float (&acc)[RW][T]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int t = 0; t < T; ++t)
        if (lane == t) {
            float* d = dst + (long long)pr[t] * n_cols + row0;
            if constexpr (RW == 4) __stcg(reinterpret_cast<float4*>(d), make_float4(acc[0][t], acc[1][t], acc[2][t], acc[3][t]));
            else if constexpr (RW == 2) __stcg(reinterpret_cast<float2*>(d), make_float2(acc[0][t], acc[1][t]));
            else {
#pragma unroll
                for (int r = 0; r < RW; ++r) __stcg(d + r, acc[r][t]);
            }
        }
}

// one warp: the lanes' stores are published by lane 0's acquire-release add on the counter (after the
// warp's sync, as the chain's group counters do); true on every lane of the warp whose add completed
// the count, which then reads the others' stores with __ldcg after the warp's sync
__device__ __forceinline__ bool moe_arrive(int* counter, int count) {
    __syncwarp();
    int last = 0;
    if ((threadIdx.x & 31) == 0) {
        int old;
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
        last = old == count - 1;
    }
    last = __shfl_sync(0xffffffffu, last, 0);
    __syncwarp();
    return last != 0;
}

template <int FMT>
__global__ void __launch_bounds__(kMoeThreads, kMoeMinBlocks) moe_gateup_kernel(const MoeParams P) {
    __shared__ MoeRoute R;
    __shared__ uint2 grid[smem_grid_format<FMT>() ? 256 : 1];
    // programmatic dependent launch: the next kernel may launch now; the routing ids, the activation
    // and the counters are read only after the previous kernel has completed (the codebook is a constant)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if constexpr (smem_grid_format<FMT>()) load_grid<FMT>(grid);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    moe_route(P, R);
    MvParams A{};
    A.xq = P.xq; A.xq2 = P.xq2; A.xd = P.xd; A.xs = P.xs; A.n_in = P.dim;
    const long long row_bytes = (long long)(P.dim / block_values(FMT)) * block_bytes(FMT);
    const int groups = P.ff / 32;
    const int lane = threadIdx.x & 31;
    const long long units = (long long)R.nu * groups * kMoeQuads;
    const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
    // unit -> (expert u, group g, quad q): the first half of the quads gate rows 32 g + RW q.., the
    // second half up rows
    constexpr int kHalf = kMoeQuads / 2;
    auto rows_of = [&](long long it, int& u, int& g, int& q) -> const uint8_t* {
        q = int(it % kMoeQuads);
        const long long item = it / kMoeQuads;
        u = int(item / groups);
        g = int(item % groups);
        const long long e = R.expert[u];
        const uint8_t* m = q < kHalf ? P.gate + e * P.gate_per : P.up + e * P.up_per;
        return m + (32LL * g + kMoeRW * (q % kHalf)) * row_bytes;
    };
    long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (it < units && lane == 0) {
        int u, g, q;
        moe_prefetch(rows_of(it, u, g, q), kMoeRW * row_bytes);
    }
    for (; it < units; it += nwarps) {
        int u, g, q;
        const uint8_t* base = rows_of(it, u, g, q);
        if (it + nwarps < units && lane == 0) {
            int u2, g2, q2;
            moe_prefetch(rows_of(it + nwarps, u2, g2, q2), kMoeRW * row_bytes);
        }
        const int ne = R.start[u + 1] - R.start[u];
        const int row0 = 32 * g + kMoeRW * (q % kHalf);
        for (int c0 = 0; c0 < ne; c0 += kMoeChunk) {
            const short* pr = R.pair + R.start[u] + c0;
            moe_with_t(min(kMoeChunk, ne - c0), [&](auto c) {
                constexpr int T = decltype(c)::value;
                Tok<T> tk;
#pragma unroll
                for (int t = 0; t < T; ++t) tk.tb[t] = (long long)(pr[t] / P.k) * P.dim;
                float acc[kMoeRW][T];
                moe_rows<FMT, T, kMoeRW>(base - (long long)row0 * row_bytes, row_bytes, row0, P.dim, A, tk, acc, grid);
                moe_store<T, kMoeRW>(q < kHalf ? P.gs : P.us, P.ff, row0, pr, acc);
            });
        }
        // the group's last quad: silu(g) * u for every pair of the expert, quantised (lane = value)
        if (moe_arrive(P.gu_done + (long long)u * groups + g, kMoeQuads)) {
            for (int c0 = 0; c0 < ne; c0 += 4) {        // four pairs' sums in flight at a time
                float gv[4], uv[4];
                long long o[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    o[c] = c0 + c < ne ? (long long)R.pair[R.start[u] + c0 + c] * P.ff + 32 * g + lane : 0;
                    gv[c] = c0 + c < ne ? __ldcg(P.gs + o[c]) : 0.f;
                    uv[c] = c0 + c < ne ? __ldcg(P.us + o[c]) : 0.f;
                }
#pragma unroll
                for (int c = 0; c < 4; ++c)
                    if (c0 + c < ne) quantize_group(gv[c] / (1.0f + expf(-gv[c])) * uv[c], o[c], P.aq, P.aq2, P.ad, P.as);
            }
        }
    }
}

template <int FMT>
__global__ void __launch_bounds__(kMoeThreads, kMoeMinBlocks) moe_down_kernel(const MoeParams P) {
    __shared__ MoeRoute R;
    __shared__ uint2 grid[smem_grid_format<FMT>() ? 256 : 1];
    // programmatic dependent launch: the next kernel may launch now; the routing ids, the activation
    // and the counters are read only after the previous kernel has completed (the codebook is a constant)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if constexpr (smem_grid_format<FMT>()) load_grid<FMT>(grid);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    moe_route(P, R);
    MvParams A{};
    A.xq = P.aq; A.xq2 = P.aq2; A.xd = P.ad; A.xs = P.as; A.n_in = P.ff;
    const long long row_bytes = (long long)(P.ff / block_values(FMT)) * block_bytes(FMT);
    const int blocks = P.dim / kMoeRW;
    const int lane = threadIdx.x & 31;
    if (R.nu == 0) {                                      // nothing valid: zeros
        for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)P.L * P.dim;
             i += (long long)gridDim.x * blockDim.x)
            P.out[i] = 0.f;
        return;
    }
    const long long units = (long long)R.nu * blocks;
    const long long nwarps = (long long)gridDim.x * (blockDim.x >> 5);
    // unit -> (expert u, block rb): consecutive units walk one expert's rows
    auto rows_of = [&](long long it, int& u, int& rb) -> const uint8_t* {
        u = int(it / blocks);
        rb = int(it % blocks);
        return P.down + (long long)R.expert[u] * P.down_per + (long long)kMoeRW * rb * row_bytes;
    };
    long long it = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (it < units && lane == 0) {
        int u, rb;
        moe_prefetch(rows_of(it, u, rb), kMoeRW * row_bytes);
    }
    for (; it < units; it += nwarps) {
        int u, rb;
        const uint8_t* base = rows_of(it, u, rb);
        if (it + nwarps < units && lane == 0) {
            int u2, rb2;
            moe_prefetch(rows_of(it + nwarps, u2, rb2), kMoeRW * row_bytes);
        }
        const int ne = R.start[u + 1] - R.start[u];
        const int row0 = kMoeRW * rb;
        for (int c0 = 0; c0 < ne; c0 += kMoeChunk) {
            const short* pr = R.pair + R.start[u] + c0;
            moe_with_t(min(kMoeChunk, ne - c0), [&](auto c) {
                constexpr int T = decltype(c)::value;
                Tok<T> tk;
#pragma unroll
                for (int t = 0; t < T; ++t) tk.tb[t] = (long long)pr[t] * P.ff;
                float acc[kMoeRW][T];
                moe_rows<FMT, T, kMoeRW>(base - (long long)row0 * row_bytes, row_bytes, row0, P.ff, A, tk, acc, grid);
                moe_store<T, kMoeRW>(P.y, P.dim, row0, pr, acc);
            });
        }
        // the block's last expert: out[t][row] = sum over the token's slots, in slot order, of w * y
        if (moe_arrive(P.d_done + rb, R.nu)) {
            for (int i = lane; i < P.L * kMoeRW; i += 32) {
                const int t = i / kMoeRW, r = row0 + i % kMoeRW;
                float v = 0.f;
                for (int j0 = 0; j0 < P.k; j0 += 8) {     // eight slots' loads in flight, added in slot order
                    float yv[8], wv[8];
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int p = t * P.k + j0 + jj;
                        const bool ok = j0 + jj < P.k && R.ex[p] >= 0;
                        yv[jj] = ok ? __ldcg(P.y + (long long)p * P.dim + r) : 0.f;
                        wv[jj] = ok ? P.wts[p] : 0.f;
                    }
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int p = t * P.k + j0 + jj;
                        if (j0 + jj < P.k && R.ex[p] >= 0) v = __fadd_rn(v, __fmul_rn(wv[jj], yv[jj]));   // no contraction
                    }
                }
                P.out[(long long)t * P.dim + r] = v;
            }
        }
    }
}

}  // namespace qmv
