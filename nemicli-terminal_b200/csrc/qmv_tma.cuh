// Single-token matvec with bulk-copy (TMA) staged weight tiles — the batch-1 hot path on sm_100a.
//
// A persistent CTA per SM: one producer warp streams tiles of R consecutive weight rows from HBM
// into a ring of shared-memory stages with cp.async.bulk (one copy per tile, completion counted on
// an mbarrier); NCW consumer warps hold their slice of the activation input in registers for the
// whole launch and read the weights from shared memory.  A row's units (32 or 64 values) are split
// across a team of G lanes (unit u -> lane u % G, then u + G, ...); 32*NCW / G teams take rows side by
// side.  Teams wider than a warp combine their partial sums through shared memory behind a named
// barrier of their own.  No TMA multicast is used.
//
// Every wait on an mbarrier is bounded in time (~1 s of %globaltimer): on expiry the waiter sets
// DEV_TIMEOUT in the status word, keeps stepping through the remaining barriers without work, and
// the producer drains the copies it issued before the CTA leaves.
#pragma once
#include "qmv_common.cuh"
#include "qmv_kernels.cuh"

namespace qmv {

constexpr int kMaxJobs = 4;
constexpr unsigned long long kWaitNs = 1000000000ull;    // bound of every mbarrier wait
enum : int { DEV_TIMEOUT = 2 };

struct TmaParams {
    // slots: either dense jobs (ids == nullptr; w/y/n_out per job, all sharing the activation) or the
    // k experts picked by ids (w[0] = expert tensor or address table, y[0] = [slot][n_out])
    const uint8_t* w[kMaxJobs];
    float* y[kMaxJobs];
    int n_out[kMaxJobs];
    long long row_start[kMaxJobs + 1]; // dense jobs: first global row of each job (prefix sums of n_out)
    int n_jobs;
    const long long* ids;
    long long per_expert;             // >= 0: expert stride in bytes; < 0: w[0] is an address table
    long long n_exp;
    int x_group;                      // slot j reads activation row j / x_group (experts)
    const int8_t* xq;
    const int8_t* xq2;
    const float* xd;
    const float* xs;
    long long row_bytes;              // multiple of 16
    int n_in;
    int rows_per_tile;                // R
    int stages;
    long long total_rows;             // rows of all jobs (dense) or k * n_out (experts)
    int* status;
    int32_t* s;                       // sums mode (test hook): int32 sums per (row, sum unit)
    int32_t* s2;
    const void* x;                    // fused quantisation (XF != 0): the raw activation row, fp32 or bf16
    // fused RMS norm (XF == 1 and nw set; the arithmetic and sum order of the norm kernel, qmv_aux.cu):
    // v = x (+ nrs * nr, written to nh, a slice per CTA), quantised input v * rsqrt(mean(v^2) + neps) * nw
    const float* nr;
    const float* nw;
    float* nh;
    float nrs, neps;
    // epilogue producer (dense jobs, teams wider than a warp): the next matvec's activation input from
    // this launch's outputs.  A counter per 32-row group (ep_cnt, zero before the call, zero again after
    // it) counts the group's rows as CTAs write them; the CTA that completes a group forms its input:
    //   ep_kind 1: job ep_j0's outputs quantised (quant_q8's arithmetic)
    //   ep_kind 2: a = SiLU(job ep_j0) * job ep_j1 (act_q8's arithmetic, written to ep_a), quantised
    int ep_kind, ep_j0, ep_j1;
    int* ep_cnt;
    int8_t* ep_xq;
    int8_t* ep_xq2;
    float* ep_xd;
    float* ep_xs;
    float* ep_a;
};

// warp w of nw, after the rows [row0, row0 + rows) of job `job` are in y (all of this CTA's consumer
// threads' stores ordered before by a barrier): count them per 32-row group (the warps take the
// groups in turn, so their counter round trips overlap); for each group this completes, form its part
// of the next input (see TmaParams ep_*)
__device__ __forceinline__ void ep_groups(const TmaParams& P, int job, int row0, int rows, int w, int nw) {
    if (P.ep_kind == 0 || rows <= 0 || (job != P.ep_j0 && job != P.ep_j1)) return;
    const int lane = threadIdx.x & 31;
    const int need = P.ep_kind == 2 ? 64 : 32;
    for (int g = (row0 >> 5) + w; g <= (row0 + rows - 1) >> 5; g += nw) {
        const int a = max(row0, 32 * g), b = min(row0 + rows, 32 * g + 32);
        int last = 0;
        if (lane == 0) {
            int old;
            asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(P.ep_cnt + g), "r"(b - a) : "memory");
            last = old + (b - a) == need;
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        __syncwarp();                                    // lane 0's acquire before every lane's loads
        if (!last) continue;
        const int i = 32 * g + lane;
        float v = __ldcg(P.y[P.ep_j0] + i);
        if (P.ep_kind == 2) {
            v = act_value(v, __ldcg(P.y[P.ep_j1] + i), true, 0);
            P.ep_a[i] = v;
        }
        quantize_group(v, i, P.ep_xq, P.ep_xq2, P.ep_xd, P.ep_xs);
        if (lane == 0) P.ep_cnt[g] = 0;                  // ready for the next call
    }
}

// ---- shared-memory access -----------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16u(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds8u(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u8 %0, [%1];" : "=h"(v) : "r"(a));
    return v & 0xFFu;
}
// 16 / 8 bytes at a 2-byte aligned shared address (aligned words + funnel shifts; the extra word
// read past the end stays inside the CTA's shared memory: stages are followed by other buffers)
__device__ __forceinline__ uint4 lds16_a2(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(b), w1 = lds32(b + 4), w2 = lds32(b + 8), w3 = lds32(b + 12), w4 = lds32(b + 16);
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh), __funnelshift_r(w2, w3, sh),
                      __funnelshift_r(w3, w4, sh));
}
__device__ __forceinline__ uint2 lds8_a2(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    const uint32_t w0 = lds32(b), w1 = lds32(b + 4), w2 = lds32(b + 8);
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

// ---- mbarriers and bulk copies ------------------------------------------------------------------

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" :: "r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
    return ok != 0;
}
// try_wait that lets the hardware suspend the warp until the phase completes (up to ~hint ns)
__device__ __forceinline__ bool mbar_try_suspend(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
                 : "=r"(ok) : "r"(bar), "r"(parity), "r"(1000000u) : "memory");
    return ok != 0;
}
// bounded wait: true when the phase with this parity completed, false after ~kWaitNs
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        if (mbar_try_suspend(bar, parity)) return true;
        if (global_ns() - t0 > kWaitNs) return false;
    }
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(threads) : "memory");
}

// exact float of an integer 0 <= v < 2^23 without the conversion unit: the bits of 2^23 + v, minus 2^23
__device__ __forceinline__ float small_u2f(uint32_t v) { return __uint_as_float(0x4B000000u | v) - 8388608.0f; }

// unsigned bytes of a times signed bytes of b, plus c
__device__ __forceinline__ int dp4us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dot4(const uint32_t (&w)[4], const int4& x) {
    return dp4(w[3], x.w, dp4(w[2], x.z, dp4(w[1], x.y, dp4(w[0], x.x, 0))));
}
__device__ __forceinline__ int dot4us(const uint32_t (&w)[4], const int4& x) {
    return dp4us(w[3], x.w, dp4us(w[2], x.z, dp4us(w[1], x.y, dp4us(w[0], x.x, 0))));
}

// ---- per-format units ---------------------------------------------------------------------------
//
// A unit is the piece of a row one lane takes: VPU values, with NS scale groups.
//   Q4_K    64 values: the 32 qs bytes 32p..32p+31 of superblock b (sub-blocks 2p low, 2p+1 high nibbles)
//   Q6_K    64 values: positions 16h..16h+15 of half n of superblock b in all four 32-value groups
//           (ql bytes 64n+16h.., 64n+32+16h.., qh bytes 128+32n+16h..: one qh load serves four groups)
//   Q4_0    32 values: one block
//   Q8_0    32 values: one block
//   TQ2_0   32 values: qs bytes 32n+8j..+7 of superblock b: 8 values of each of the four groups of half n
//   IQ2_XXS 32 values: one sub-block (4 codebook entries)

template <int FMT> struct UnitTraits { static constexpr int VPU = 32, NS = 1, NQ = 2; };
template <> struct UnitTraits<F_Q4_K> { static constexpr int VPU = 64, NS = 2, NQ = 4; };
template <> struct UnitTraits<F_Q5_K> { static constexpr int VPU = 64, NS = 2, NQ = 4; };
template <> struct UnitTraits<F_Q3_K> { static constexpr int VPU = 32, NS = 2, NQ = 2; };   // two 16-value scales
template <> struct UnitTraits<F_IQ2_XS> { static constexpr int VPU = 32, NS = 2, NQ = 2; };
template <> struct UnitTraits<F_IQ2_S> { static constexpr int VPU = 32, NS = 2, NQ = 2; };
template <> struct UnitTraits<F_Q2_K> { static constexpr int VPU = 32, NS = 2, NQ = 2; };
template <> struct UnitTraits<F_Q6_K> { static constexpr int VPU = 64, NS = 4, NQ = 4; };
// Q6_K with 32-value units (ql bytes 64n+16j..+15 of superblock b: 16 values of group j/2 and of j/2 + 2):
// a smaller activation footprint, for the decode chain's register budget.  Internal tag only.
constexpr int F_Q6_K_U32 = 0x100 | F_Q6_K;
template <> struct UnitTraits<F_Q6_K_U32> { static constexpr int VPU = 32, NS = 2, NQ = 2; };
template <> struct UnitTraits<F_TQ2_0> { static constexpr int VPU = 32, NS = 4, NQ = 2; };

template <int FMT>
struct Act {                              // the activation of one unit, in registers
    int4 q[UnitTraits<FMT>::NQ];          // xq bytes
    int4 r[UnitTraits<FMT>::NQ];          // xq2 bytes
    float d[UnitTraits<FMT>::NS];         // xd / 254 of each scale group
    float s[UnitTraits<FMT>::NS];         // xs of each group (0 where another lane applies the offset)
    int sq[FMT == F_Q6_K ? 4 : FMT == F_Q6_K_U32 ? 2 : 1];   // Q6_K: sum of the 16 xq of each group
    int sr[FMT == F_Q6_K ? 4 : FMT == F_Q6_K_U32 ? 2 : 1];   //       sum of the 16 xq2 of each group
    int kk[FMT == F_Q6_K ? 4 : 1];        //       32 * (254 sq + sr): the -32 of 254 S + S2
};

// activation sources: SRC_SMEM shared memory; SRC_NC global through the read-only path (inputs that
// no kernel in flight writes); SRC_CG global through L2 only (written earlier in the same launch)
enum : int { SRC_SMEM = 0, SRC_NC = 1, SRC_CG = 2 };
template <int SRC>
__device__ __forceinline__ int4 ldq16(const int8_t* p) {
    if constexpr (SRC == SRC_NC) return __ldg(reinterpret_cast<const int4*>(p));
    if constexpr (SRC == SRC_CG) return __ldcg(reinterpret_cast<const int4*>(p));
    return *reinterpret_cast<const int4*>(p);
}
template <int SRC>
__device__ __forceinline__ int2 ldq8(const int8_t* p) {
    if constexpr (SRC == SRC_NC) return __ldg(reinterpret_cast<const int2*>(p));
    if constexpr (SRC == SRC_CG) return __ldcg(reinterpret_cast<const int2*>(p));
    return *reinterpret_cast<const int2*>(p);
}
template <int SRC, bool SCALES>
__device__ __forceinline__ float ldf(const float* p, int i) {
    if constexpr (!SCALES) return 0.f;
    if constexpr (SRC == SRC_NC) return __ldg(p + i);
    if constexpr (SRC == SRC_CG) return __ldcg(p + i);
    return p[i];
}

// xq/xq2/xd/xs point at the start of the activation row (in memory of kind SRC).  SCALES = false
// (the int32-sums test hook) reads xq/xq2 only: xd/xs may be null.
template <int FMT, bool SCALES, int GLOBAL = SRC_NC>
__device__ __forceinline__ void load_act(Act<FMT>& a, int u, const int8_t* xq, const int8_t* xq2, const float* xd,
                                         const float* xs) {
    constexpr int NS = UnitTraits<FMT>::NS;
#pragma unroll
    for (int i = 0; i < NS; ++i) a.d[i] = a.s[i] = 0.f;
    if constexpr (FMT == F_Q4_0 || FMT == F_Q8_0 || FMT == F_IQ2_XXS || FMT == F_IQ4_XS || FMT == F_MXFP4 ||
                  FMT == F_IQ3_S || FMT == F_IQ3_XXS || FMT == F_Q4_1 || FMT == F_Q5_0 || FMT == F_Q5_1 ||
                  FMT == F_IQ4_NL || bits_format(FMT)) {
        const int o = 32 * u;
        a.q[0] = ldq16<GLOBAL>(xq + o); a.q[1] = ldq16<GLOBAL>(xq + o + 16);
        a.r[0] = ldq16<GLOBAL>(xq2 + o); a.r[1] = ldq16<GLOBAL>(xq2 + o + 16);
        a.d[0] = ldf<GLOBAL, SCALES>(xd, u) * kInv254;
        if (FMT == F_Q4_0 || FMT == F_Q4_1 || FMT == F_Q5_0 || FMT == F_Q5_1 || bits_format(FMT)) a.s[0] = ldf<GLOBAL, SCALES>(xs, u);
        if constexpr (FMT == F_Q2_0 || FMT == F_PQ2_0) {       // the order of the 2-bit codes
            a.q[0] = byte_transpose(a.q[0]); a.q[1] = byte_transpose(a.q[1]);
            a.r[0] = byte_transpose(a.r[0]); a.r[1] = byte_transpose(a.r[1]);
        }
    } else if constexpr (FMT == F_Q4_K || FMT == F_Q5_K) {
        const int b = u >> 2, p = u & 3, o = b * 256 + 64 * p;
        a.q[0] = ldq16<GLOBAL>(xq + o); a.q[1] = ldq16<GLOBAL>(xq + o + 16);
        a.q[2] = ldq16<GLOBAL>(xq + o + 32); a.q[3] = ldq16<GLOBAL>(xq + o + 48);
        a.r[0] = ldq16<GLOBAL>(xq2 + o); a.r[1] = ldq16<GLOBAL>(xq2 + o + 16);
        a.r[2] = ldq16<GLOBAL>(xq2 + o + 32); a.r[3] = ldq16<GLOBAL>(xq2 + o + 48);
        a.d[0] = ldf<GLOBAL, SCALES>(xd, b * 8 + 2 * p) * kInv254;
        a.d[1] = ldf<GLOBAL, SCALES>(xd, b * 8 + 2 * p + 1) * kInv254;
        a.s[0] = ldf<GLOBAL, SCALES>(xs, b * 8 + 2 * p);
        a.s[1] = ldf<GLOBAL, SCALES>(xs, b * 8 + 2 * p + 1);
    } else if constexpr (FMT == F_Q3_K || iq2x_format(FMT) || FMT == F_Q2_K) {
        const int o = 32 * u;
        a.q[0] = ldq16<GLOBAL>(xq + o); a.q[1] = ldq16<GLOBAL>(xq + o + 16);
        a.r[0] = ldq16<GLOBAL>(xq2 + o); a.r[1] = ldq16<GLOBAL>(xq2 + o + 16);
        a.d[0] = a.d[1] = ldf<GLOBAL, SCALES>(xd, u) * kInv254;
        if constexpr (FMT == F_Q2_K) {
            // the minimum's activation: (xd / 254) (254 sum xq + sum xq2) of each 16-value half
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                const int4 x = a.q[g], y = a.r[g];
                const int sq = dp4(0x01010101u, x.w, dp4(0x01010101u, x.z, dp4(0x01010101u, x.y, dp4(0x01010101u, x.x, 0))));
                const int sr = dp4(0x01010101u, y.w, dp4(0x01010101u, y.z, dp4(0x01010101u, y.y, dp4(0x01010101u, y.x, 0))));
                a.s[g] = a.d[g] * float(254 * sq + sr);
            }
        }
    } else if constexpr (FMT == F_Q6_K_U32) {
        const int b = u >> 3, q = u & 7, n = q >> 2, j = q & 3, A = j >> 1, B = A + 2, o = b * 256 + 128 * n + 16 * (j & 1);
        a.q[0] = ldq16<GLOBAL>(xq + o + 32 * A); a.q[1] = ldq16<GLOBAL>(xq + o + 32 * B);
        a.r[0] = ldq16<GLOBAL>(xq2 + o + 32 * A); a.r[1] = ldq16<GLOBAL>(xq2 + o + 32 * B);
        a.d[0] = ldf<GLOBAL, SCALES>(xd, b * 8 + 4 * n + A) * kInv254;
        a.d[1] = ldf<GLOBAL, SCALES>(xd, b * 8 + 4 * n + B) * kInv254;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
            const int4 x = a.q[g], y = a.r[g];
            a.sq[g] = dp4(0x01010101u, x.w, dp4(0x01010101u, x.z, dp4(0x01010101u, x.y, dp4(0x01010101u, x.x, 0))));
            a.sr[g] = dp4(0x01010101u, y.w, dp4(0x01010101u, y.z, dp4(0x01010101u, y.y, dp4(0x01010101u, y.x, 0))));
        }
    } else if constexpr (FMT == F_Q6_K) {
        const int b = u >> 2, n = (u >> 1) & 1, h = u & 1, o = b * 256 + 128 * n + 16 * h;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            a.q[g] = ldq16<GLOBAL>(xq + o + 32 * g);
            a.r[g] = ldq16<GLOBAL>(xq2 + o + 32 * g);
            a.d[g] = ldf<GLOBAL, SCALES>(xd, b * 8 + 4 * n + g) * kInv254;
            const int4 x = a.q[g], y = a.r[g];
            a.sq[g] = dp4(0x01010101u, x.w, dp4(0x01010101u, x.z, dp4(0x01010101u, x.y, dp4(0x01010101u, x.x, 0))));
            a.sr[g] = dp4(0x01010101u, y.w, dp4(0x01010101u, y.z, dp4(0x01010101u, y.y, dp4(0x01010101u, y.x, 0))));
            a.kk[g] = 32 * (254 * a.sq[g] + a.sr[g]);
        }
    } else {   // TQ2_0
        const int b = u >> 3, q = u & 7, n = q >> 2, j = q & 3, o = b * 256 + 128 * n + 8 * j;
        const int2 g0 = ldq8<GLOBAL>(xq + o), g1 = ldq8<GLOBAL>(xq + o + 32), g2 = ldq8<GLOBAL>(xq + o + 64),
                   g3 = ldq8<GLOBAL>(xq + o + 96);
        const int2 h0 = ldq8<GLOBAL>(xq2 + o), h1 = ldq8<GLOBAL>(xq2 + o + 32), h2 = ldq8<GLOBAL>(xq2 + o + 64),
                   h3 = ldq8<GLOBAL>(xq2 + o + 96);
        a.q[0] = make_int4(g0.x, g0.y, g1.x, g1.y); a.q[1] = make_int4(g2.x, g2.y, g3.x, g3.y);
        a.r[0] = make_int4(h0.x, h0.y, h1.x, h1.y); a.r[1] = make_int4(h2.x, h2.y, h3.x, h3.y);
        // a.d[g] carries 4^-g (exact): unit_dot takes group g's codes in place, 4^g times their value;
        // a.s[0] the four groups' xs (applied by one lane of the four that share the groups)
#pragma unroll
        for (int g = 0; g < 4; ++g) a.d[g] = ldf<GLOBAL, SCALES>(xd, b * 8 + 4 * n + g) * (kInv254 / float(1 << (2 * g)));
        if (j == 0)
            a.s[0] = (ldf<GLOBAL, SCALES>(xs, b * 8 + 4 * n) + ldf<GLOBAL, SCALES>(xs, b * 8 + 4 * n + 1)) +
                     (ldf<GLOBAL, SCALES>(xs, b * 8 + 4 * n + 2) + ldf<GLOBAL, SCALES>(xs, b * 8 + 4 * n + 3));
    }
}

// Integer stage of one unit: weight codes of the staged row at shared address `rs` times xq and xq2.
// s[k], u[k]: int32 sums of scale group k; wsc[k]: weight scale; off[k]: weight offset (times xs).
template <int FMT>
struct UnitSums {
    int s[UnitTraits<FMT>::NS], u[UnitTraits<FMT>::NS];
    float wsc[UnitTraits<FMT>::NS], off[UnitTraits<FMT>::NS];
};
// Q4_K keeps its 6-bit scales / mins as integers and applies d, dmin once per unit
template <>
struct UnitSums<F_Q4_K> {
    int s[2], u[2], isc[2];
    uint32_t imn[2];
    float d, dm;
};
template <>
struct UnitSums<F_Q5_K> : UnitSums<F_Q4_K> {};

// 6-bit scales / mins of sub-blocks 2p, 2p + 1 from a K-quant header word hd (quant.py:99-108): the two
// scale bytes and the two min bytes of the pair gathered by byte permutes (sub-blocks 0..3: low 6 bits of
// bytes j and j + 4 of the 12; 4..7: the nibbles of byte j + 4 with the top two bits of bytes j - 4 and
// j), no branch on p
__device__ __forceinline__ void kquant_scales(const uint4& hd, int p, int (&isc)[2], uint32_t (&imn)[2]) {
    const uint32_t b = 2u * uint32_t(p & 1);                            // first byte of the pair in its word
    const uint32_t yz = __byte_perm(hd.y, hd.z, b | ((b + 1) << 4) | ((b + 4) << 8) | ((b + 5) << 12));
    const uint32_t ww = __byte_perm(hd.w, 0u, b | ((b + 1) << 4) | (b << 8) | ((b + 1) << 12));
    const uint32_t lo = yz & 0x3F3F3F3Fu;
    const uint32_t hi = (ww & 0x00000F0Fu) | ((ww >> 4) & 0x0F0F0000u) | ((yz >> 2) & 0x30303030u);
    const uint32_t pk = p < 2 ? lo : hi;                                // [sc0, sc1, m0, m1]
    isc[0] = int(pk & 0xFFu);
    isc[1] = int((pk >> 8) & 0xFFu);
    imn[0] = (pk >> 16) & 0xFFu;
    imn[1] = pk >> 24;
}

// unsigned 6-bit codes of a Q6_K unit (w[g][i]: 4 codes of group g, positions 16h + 4i..): group g's low
// four bits from ql (low nibbles for g = 0, 1, high for g = 2, 3), bits 4..5 from qh bits 2g..2g+1; the
// -32 of every code is taken off with the activation sums
__device__ __forceinline__ void q6k_codes(uint32_t sb, int n, int h, uint32_t (&w)[4][4]) {
    const uint4 l0 = lds16_a2(sb + 64 * n + 16 * h), l1 = lds16_a2(sb + 64 * n + 32 + 16 * h);
    const uint4 qh = lds16_a2(sb + 128 + 32 * n + 16 * h);
    const uint32_t A[4] = {l0.x, l0.y, l0.z, l0.w}, B[4] = {l1.x, l1.y, l1.z, l1.w}, H[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        w[0][i] = (A[i] & 0x0F0F0F0Fu) | ((H[i] << 4) & 0x30303030u);
        w[1][i] = (B[i] & 0x0F0F0F0Fu) | ((H[i] << 2) & 0x30303030u);
        w[2][i] = ((A[i] >> 4) & 0x0F0F0F0Fu) | (H[i] & 0x30303030u);
        w[3][i] = ((B[i] >> 4) & 0x0F0F0F0Fu) | ((H[i] >> 2) & 0x30303030u);
    }
}

template <int FMT>
__device__ __forceinline__ void unit_sums(uint32_t rs, int u, const Act<FMT>& a, UnitSums<FMT>& o, const uint2* grid) {
    if constexpr (FMT == F_Q4_K) {
        const int b = u >> 2, p = u & 3;
        const uint32_t sb = rs + b * 144;
        const uint4 hd = lds128(sb), v0 = lds128(sb + 16 + 32 * p), v1 = lds128(sb + 32 + 32 * p);
        const uint32_t l0[4] = {v0.x & 0x0F0F0F0Fu, v0.y & 0x0F0F0F0Fu, v0.z & 0x0F0F0F0Fu, v0.w & 0x0F0F0F0Fu};
        const uint32_t l1[4] = {v1.x & 0x0F0F0F0Fu, v1.y & 0x0F0F0F0Fu, v1.z & 0x0F0F0F0Fu, v1.w & 0x0F0F0F0Fu};
        const uint32_t h0[4] = {v0.x & 0xF0F0F0F0u, v0.y & 0xF0F0F0F0u, v0.z & 0xF0F0F0F0u, v0.w & 0xF0F0F0F0u};
        const uint32_t h1[4] = {v1.x & 0xF0F0F0F0u, v1.y & 0xF0F0F0F0u, v1.z & 0xF0F0F0F0u, v1.w & 0xF0F0F0F0u};
        // sub-block 2p: low nibbles of the 32 bytes; 2p+1: high nibbles (16 x the nibble, shifted out below)
        o.s[0] = dot4(l1, a.q[1]) + dot4(l0, a.q[0]);
        o.u[0] = dot4(l1, a.r[1]) + dot4(l0, a.r[0]);
        o.s[1] = (dot4us(h1, a.q[3]) + dot4us(h0, a.q[2])) >> 4;
        o.u[1] = (dot4us(h1, a.r[3]) + dot4us(h0, a.r[2])) >> 4;
        kquant_scales(hd, p, o.isc, o.imn);
        o.d = h2f(hd.x & 0xFFFFu);
        o.dm = h2f(hd.x >> 16);
    } else if constexpr (FMT == F_Q5_K) {
        // Q5_K (quant.py:123-137): the Q4_K header, qh[32] at 16, qs[128] at 48; the unsigned 5-bit code
        // of value i of sub-block 2p (2p+1) is the low (high) nibble of qs[32p + i] with bit 2p (2p+1)
        // of qh[i] as bit 4
        const int b = u >> 2, p = u & 3;
        const uint32_t sb = rs + b * 176;
        const uint4 hd = lds128(sb), q0 = lds128(sb + 16), q1 = lds128(sb + 32);
        const uint4 v0 = lds128(sb + 48 + 32 * p), v1 = lds128(sb + 64 + 32 * p);
        const uint32_t H0[4] = {q0.x, q0.y, q0.z, q0.w}, H1[4] = {q1.x, q1.y, q1.z, q1.w};
        const uint32_t V0[4] = {v0.x, v0.y, v0.z, v0.w}, V1[4] = {v1.x, v1.y, v1.z, v1.w};
        uint32_t l0[4], l1[4], g0[4], g1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            l0[i] = (V0[i] & 0x0F0F0F0Fu) | (((H0[i] >> (2 * p)) & 0x01010101u) << 4);
            l1[i] = (V1[i] & 0x0F0F0F0Fu) | (((H1[i] >> (2 * p)) & 0x01010101u) << 4);
            g0[i] = ((V0[i] >> 4) & 0x0F0F0F0Fu) | (((H0[i] >> (2 * p + 1)) & 0x01010101u) << 4);
            g1[i] = ((V1[i] >> 4) & 0x0F0F0F0Fu) | (((H1[i] >> (2 * p + 1)) & 0x01010101u) << 4);
        }
        o.s[0] = dot4(l1, a.q[1]) + dot4(l0, a.q[0]);
        o.u[0] = dot4(l1, a.r[1]) + dot4(l0, a.r[0]);
        o.s[1] = dot4(g1, a.q[3]) + dot4(g0, a.q[2]);
        o.u[1] = dot4(g1, a.r[3]) + dot4(g0, a.r[2]);
        kquant_scales(hd, p, o.isc, o.imn);
        o.d = h2f(hd.x & 0xFFFFu);
        o.dm = h2f(hd.x >> 16);
    } else if constexpr (FMT == F_Q6_K_U32) {
        const int b = u >> 3, q = u & 7, n = q >> 2, j = q & 3, A = j >> 1, B = A + 2, l0 = 16 * (j & 1);
        const uint32_t sb = rs + b * 210;
        const uint4 ql = lds16_a2(sb + 64 * n + 16 * j), qh = lds16_a2(sb + 128 + 32 * n + l0);
        const uint32_t L[4] = {ql.x, ql.y, ql.z, ql.w}, H[4] = {qh.x, qh.y, qh.z, qh.w};
        // unsigned 6-bit codes: group A = low nibble | qh bits 2A..2A+1 moved to bits 4..5, group A + 2 =
        // high nibble | qh bits 2A+4..2A+5; the -32 of every code is subtracted with the activation sums
        const int shA = 4 - 2 * A, shB = 2 * A;
        uint32_t wa[4], wb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wa[i] = (L[i] & 0x0F0F0F0Fu) | ((H[i] << shA) & 0x30303030u);
            wb[i] = ((L[i] >> 4) & 0x0F0F0F0Fu) | ((H[i] >> shB) & 0x30303030u);
        }
        o.s[0] = dot4(wa, a.q[0]) - 32 * a.sq[0];
        o.s[1] = dot4(wb, a.q[1]) - 32 * a.sq[1];
        o.u[0] = dot4(wa, a.r[0]) - 32 * a.sr[0];
        o.u[1] = dot4(wb, a.r[1]) - 32 * a.sr[1];
        const float d = h2f(lds16u(sb + 208));
        o.wsc[0] = d * float(int8_t(lds8u(sb + 192 + 8 * n + 2 * A + (j & 1))));
        o.wsc[1] = d * float(int8_t(lds8u(sb + 192 + 8 * n + 2 * B + (j & 1))));
        o.off[0] = o.off[1] = 0.f;
    } else if constexpr (FMT == F_Q6_K) {
        const int b = u >> 2, n = (u >> 1) & 1, h = u & 1;
        const uint32_t sb = rs + b * 210;
        uint32_t w[4][4];
        q6k_codes(sb, n, h, w);
        const float d = h2f(lds16u(sb + 208));
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            o.s[g] = dot4(w[g], a.q[g]) - 32 * a.sq[g];
            o.u[g] = dot4(w[g], a.r[g]) - 32 * a.sr[g];
            o.wsc[g] = d * float(int8_t(lds8u(sb + 192 + 8 * n + 2 * g + h)));
            o.off[g] = 0.f;
        }
    } else if constexpr (FMT == F_Q4_0) {
        const uint32_t bl = rs + u * 18;
        const uint4 v = lds16_a2(bl + 2);
        const uint32_t lo[4] = {v.x & 0x0F0F0F0Fu, v.y & 0x0F0F0F0Fu, v.z & 0x0F0F0F0Fu, v.w & 0x0F0F0F0Fu};
        const uint32_t hi[4] = {v.x & 0xF0F0F0F0u, v.y & 0xF0F0F0F0u, v.z & 0xF0F0F0F0u, v.w & 0xF0F0F0F0u};
        o.s[0] = dot4(lo, a.q[0]) + (dot4us(hi, a.q[1]) >> 4);
        o.u[0] = dot4(lo, a.r[0]) + (dot4us(hi, a.r[1]) >> 4);
        const float d = h2f(lds16u(bl));
        o.wsc[0] = d;
        o.off[0] = 8.0f * d;
    } else if constexpr (FMT == F_Q8_0) {
        const uint32_t bl = rs + u * 34;
        const uint4 v0 = lds16_a2(bl + 2), v1 = lds16_a2(bl + 18);
        const uint32_t w0[4] = {v0.x, v0.y, v0.z, v0.w}, w1[4] = {v1.x, v1.y, v1.z, v1.w};
        o.s[0] = dot4(w1, a.q[1]) + dot4(w0, a.q[0]);
        o.u[0] = dot4(w1, a.r[1]) + dot4(w0, a.r[0]);
        o.wsc[0] = h2f(lds16u(bl));
        o.off[0] = 0.f;
    } else if constexpr (FMT == F_TQ2_0) {
        const int b = u >> 3, q = u & 7, n = q >> 2, j = q & 3;
        const uint32_t sb = rs + b * 66;
        const uint2 c = lds8_a2(sb + 32 * n + 8 * j);
        const float d = h2f(lds16u(sb + 64));
        const int xq[8] = {a.q[0].x, a.q[0].y, a.q[0].z, a.q[0].w, a.q[1].x, a.q[1].y, a.q[1].z, a.q[1].w};
        const int xr[8] = {a.r[0].x, a.r[0].y, a.r[0].z, a.r[0].w, a.r[1].x, a.r[1].y, a.r[1].z, a.r[1].w};
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint32_t c0 = (c.x >> (2 * g)) & 0x03030303u, c1 = (c.y >> (2 * g)) & 0x03030303u;
            o.s[g] = dp4(c1, xq[2 * g + 1], dp4(c0, xq[2 * g], 0));
            o.u[g] = dp4(c1, xr[2 * g + 1], dp4(c0, xr[2 * g], 0));
            o.wsc[g] = d;
            o.off[g] = d;
        }
    } else if constexpr (FMT == F_Q4_1 || FMT == F_Q5_0 || FMT == F_Q5_1 || FMT == F_IQ4_NL) {
        constexpr int qo = FMT == F_Q4_1 ? 4 : FMT == F_Q5_0 ? 6 : FMT == F_Q5_1 ? 8 : 2;
        const uint32_t bl = rs + u * block_bytes(FMT);
        const uint4 v = lds16_a2(bl + qo);
        const uint32_t V[4] = {v.x, v.y, v.z, v.w};
        uint32_t qh = 0u;
        if constexpr (FMT == F_Q5_0) qh = lds16u(bl + 2) | (lds16u(bl + 4) << 16);
        if constexpr (FMT == F_Q5_1) qh = lds16u(bl + 4) | (lds16u(bl + 6) << 16);
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (FMT == F_IQ4_NL) {
                lo[i] = iq4nl_bytes(V[i] & 0x0F0F0F0Fu);
                hi[i] = iq4nl_bytes((V[i] >> 4) & 0x0F0F0F0Fu);
            } else {
                lo[i] = (V[i] & 0x0F0F0F0Fu) | (spread4(qh >> (4 * i)) << 4);
                hi[i] = ((V[i] >> 4) & 0x0F0F0F0Fu) | (spread4(qh >> (16 + 4 * i)) << 4);
            }
        }
        o.s[0] = dot4(hi, a.q[1]) + dot4(lo, a.q[0]);
        o.u[0] = dot4(hi, a.r[1]) + dot4(lo, a.r[0]);
        const float d = h2f(lds16u(bl));
        o.wsc[0] = d;
        o.off[0] = FMT == F_Q5_0 ? 16.0f * d : (FMT == F_Q4_1 || FMT == F_Q5_1) ? -h2f(lds16u(bl + 2)) : 0.f;
    } else if constexpr (iq2x_format(FMT)) {
        const int b = u >> 3, q = u & 7;
        const uint32_t sb = rs + b * block_bytes(FMT);
        uint32_t q0, q1 = 0u, sg = 0u, qh = 0u, scb;
        if constexpr (FMT == F_IQ2_XS) {
            const uint2 c = lds8_a2(sb + 2 + 8 * q);
            q0 = c.x;
            q1 = c.y;
            scb = lds8u(sb + 66 + q);
        } else {
            q0 = lds16u(sb + 2 + 4 * q) | (lds16u(sb + 4 + 4 * q) << 16);
            sg = lds16u(sb + 34 + 4 * q) | (lds16u(sb + 36 + 4 * q) << 16);
            qh = lds8u(sb + 66 + q);
            scb = lds8u(sb + 74 + q);
        }
        uint32_t w[8];
        iq2x_words<FMT>(q0, q1, sg, qh, w);
        const uint32_t w0[4] = {w[0], w[1], w[2], w[3]}, w1[4] = {w[4], w[5], w[6], w[7]};
        o.s[0] = dot4(w0, a.q[0]);
        o.u[0] = dot4(w0, a.r[0]);
        o.s[1] = dot4(w1, a.q[1]);
        o.u[1] = dot4(w1, a.r[1]);
        const float d = h2f(lds16u(sb));
        o.wsc[0] = d * (0.125f + 0.25f * float(scb & 15u));
        o.wsc[1] = d * (0.125f + 0.25f * float(scb >> 4));
        o.off[0] = o.off[1] = 0.f;
    } else if constexpr (FMT == F_Q2_K) {
        const int b = u >> 3, q = u & 7, n = q >> 2, s2 = 2 * (q & 3);
        const uint32_t sb = rs + b * 84;
        const uint4 q0 = lds16_a2(sb + 16 + 32 * n), q1 = lds16_a2(sb + 32 + 32 * n);
        const uint32_t w0[4] = {(q0.x >> s2) & 0x03030303u, (q0.y >> s2) & 0x03030303u, (q0.z >> s2) & 0x03030303u,
                                (q0.w >> s2) & 0x03030303u};
        const uint32_t w1[4] = {(q1.x >> s2) & 0x03030303u, (q1.y >> s2) & 0x03030303u, (q1.z >> s2) & 0x03030303u,
                                (q1.w >> s2) & 0x03030303u};
        o.s[0] = dot4(w0, a.q[0]);
        o.u[0] = dot4(w0, a.r[0]);
        o.s[1] = dot4(w1, a.q[1]);
        o.u[1] = dot4(w1, a.r[1]);
        const float d = h2f(lds16u(sb + 80)), dm = h2f(lds16u(sb + 82));
        const uint32_t sc0 = lds8u(sb + 2 * q), sc1 = lds8u(sb + 2 * q + 1);
        o.wsc[0] = d * float(sc0 & 15u);
        o.wsc[1] = d * float(sc1 & 15u);
        o.off[0] = dm * float(sc0 >> 4);
        o.off[1] = dm * float(sc1 >> 4);
    } else if constexpr (FMT == F_Q3_K) {
        const int b = u >> 3, q = u & 7, n = q >> 2, s2 = 2 * (q & 3);
        const uint32_t sb = rs + b * 110;
        const uint4 q0 = lds16_a2(sb + 32 + 32 * n), q1 = lds16_a2(sb + 48 + 32 * n);
        const uint4 h0 = lds16_a2(sb), h1 = lds16_a2(sb + 16);
        const uint32_t Q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const uint32_t H[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
        uint32_t w0[4], w1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0[i] = q3k_word((Q[i] >> s2) & 0x03030303u, (H[i] >> q) & 0x01010101u);
            w1[i] = q3k_word((Q[4 + i] >> s2) & 0x03030303u, (H[4 + i] >> q) & 0x01010101u);
        }
        o.s[0] = dot4(w0, a.q[0]);
        o.u[0] = dot4(w0, a.r[0]);
        o.s[1] = dot4(w1, a.q[1]);
        o.u[1] = dot4(w1, a.r[1]);
        const float d = h2f(lds16u(sb + 108));
#pragma unroll
        for (int k = 0; k < 2; ++k) {
            const int i = 2 * q + k;
            const int lo = int(lds8u(sb + 96 + i % 8) >> (4 * (i / 8))) & 15, hi = int(lds8u(sb + 104 + i % 4) >> (2 * (i / 4))) & 3;
            o.wsc[k] = d * float((lo | (hi << 4)) - 32);
            o.off[k] = 0.f;
        }
    } else if constexpr (bits_format(FMT)) {
        constexpr int upb = block_values(FMT) / 32;
        const int sub = u % upb;
        const uint32_t bl = rs + uint32_t(u / upb) * block_bytes(FMT);
        uint32_t w0[4], w1[4];
        if constexpr (FMT == F_Q1_0) {
            const uint32_t bits = lds16u(bl + 2 + 4 * sub) | (lds16u(bl + 4 + 4 * sub) << 16);
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                w0[2 * k] = spread4(bits >> (8 * k));
                w0[2 * k + 1] = spread4(bits >> (8 * k + 4));
                w1[2 * k] = spread4(bits >> (8 * k + 16));
                w1[2 * k + 1] = spread4(bits >> (8 * k + 20));
            }
        } else {
            const uint2 c = lds8_a2(bl + 2 + 8 * sub);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                w0[s] = (c.x >> (2 * s)) & 0x03030303u;
                w1[s] = (c.y >> (2 * s)) & 0x03030303u;
            }
        }
        o.s[0] = dot4(w1, a.q[1]) + dot4(w0, a.q[0]);
        o.u[0] = dot4(w1, a.r[1]) + dot4(w0, a.r[0]);
        const float d = h2f(lds16u(bl));
        o.wsc[0] = FMT == F_Q1_0 ? 2.0f * d : d;
        o.off[0] = d;
    } else if constexpr (FMT == F_IQ3_XXS) {
        const int b = u >> 3, q = u & 7;
        const uint32_t sb = rs + b * 98;
        const uint2 qs = lds8_a2(sb + 2 + 8 * q);
        const uint32_t aux = lds16u(sb + 66 + 4 * q) | (lds16u(sb + 68 + 4 * q) << 16);
        const uint32_t* g3 = reinterpret_cast<const uint32_t*>(grid);
        uint32_t w[8];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t s7 = (aux >> (7 * l)) & 127u;
            const uint32_t s8 = s7 | (uint32_t(__popc(s7) & 1) << 7);
            const uint32_t mlo = sign4_mask(s8), mhi = sign4_mask(s8 >> 4);
            const uint32_t word = l < 2 ? qs.x : qs.y;
            w[2 * l] = __vsub4(g3[(word >> (16 * (l & 1))) & 0xFFu] ^ mlo, mlo);
            w[2 * l + 1] = __vsub4(g3[(word >> (16 * (l & 1) + 8)) & 0xFFu] ^ mhi, mhi);
        }
        const uint32_t w0[4] = {w[0], w[1], w[2], w[3]}, w1[4] = {w[4], w[5], w[6], w[7]};
        o.s[0] = dot4(w1, a.q[1]) + dot4(w0, a.q[0]);
        o.u[0] = dot4(w1, a.r[1]) + dot4(w0, a.r[0]);
        o.wsc[0] = h2f(lds16u(sb)) * (0.25f + 0.5f * float(aux >> 28));
        o.off[0] = 0.f;
    } else if constexpr (FMT == F_IQ3_S) {
        const int b = u >> 3, q = u & 7;
        const uint32_t sb = rs + b * 110;
        const uint2 qs = lds8_a2(sb + 2 + 8 * q);
        const uint32_t qh = lds8u(sb + 66 + q);
        const uint32_t sg = lds16u(sb + 74 + 4 * q) | (lds16u(sb + 76 + 4 * q) << 16);
        const uint32_t* g3 = reinterpret_cast<const uint32_t*>(grid);
        uint32_t w0[4], w1[4];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t idx = (((l < 4 ? qs.x : qs.y) >> (8 * (l & 3))) & 0xFFu) | (((qh >> l) & 1u) << 8);
            const uint32_t m = sign4_mask(sg >> (4 * l));
            const uint32_t v = __vsub4(g3[idx] ^ m, m);
            if (l < 4) w0[l] = v; else w1[l - 4] = v;
        }
        o.s[0] = dot4(w1, a.q[1]) + dot4(w0, a.q[0]);
        o.u[0] = dot4(w1, a.r[1]) + dot4(w0, a.r[0]);
        const uint32_t ls = (lds8u(sb + 106 + (q >> 1)) >> (4 * (q & 1))) & 15u;
        o.wsc[0] = h2f(lds16u(sb)) * float(1 + 2 * int(ls));
        o.off[0] = 0.f;
    } else if constexpr (FMT == F_MXFP4) {
        const uint32_t bl = rs + u * 17;
        const uint4 v = lds16_a2(bl + 1);           // any byte offset: aligned words + funnel shifts
        const uint32_t V[4] = {v.x, v.y, v.z, v.w};
        uint32_t w0[4], w1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0[i] = mxfp4_bytes(V[i] & 0x0F0F0F0Fu);
            w1[i] = mxfp4_bytes((V[i] >> 4) & 0x0F0F0F0Fu);
        }
        o.s[0] = dot4(w1, a.q[1]) + dot4(w0, a.q[0]);
        o.u[0] = dot4(w1, a.r[1]) + dot4(w0, a.r[0]);
        o.wsc[0] = mxfp4_scale(lds8u(bl));
        o.off[0] = 0.f;
    } else if constexpr (FMT == F_IQ4_XS) {
        const int b = u >> 3, q = u & 7;
        const uint32_t sb = rs + b * 136;
        const uint4 v = lds16_a2(sb + 8 + 16 * q);
        const uint32_t V[4] = {v.x, v.y, v.z, v.w};
        uint32_t w0[4], w1[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w0[i] = iq4nl_bytes(V[i] & 0x0F0F0F0Fu);
            w1[i] = iq4nl_bytes((V[i] >> 4) & 0x0F0F0F0Fu);
        }
        o.s[0] = dot4(w1, a.q[1]) + dot4(w0, a.q[0]);
        o.u[0] = dot4(w1, a.r[1]) + dot4(w0, a.r[0]);
        const uint32_t sh = lds16u(sb + 2), sl = lds8u(sb + 4 + (q >> 1));
        const int ls = int(((sl >> (4 * (q & 1))) & 15u) | (((sh >> (2 * q)) & 3u) << 4));
        o.wsc[0] = h2f(lds16u(sb)) * float(ls - 32);
        o.off[0] = 0.f;
    } else {   // IQ2_XXS
        const int b = u >> 3, q = u & 7;
        const uint32_t sb = rs + b * 66;
        const uint2 ax = lds8_a2(sb + 2 + 8 * q);
        uint32_t w[8];
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint2 g = grid[__byte_perm(ax.x, 0u, 0x4440u + l)];      // byte l of the index word
            const uint32_t s7 = (ax.y >> (7 * l)) & 127u;
            const uint32_t s8 = s7 | ((uint32_t(__popc(s7)) << 7) & 0x80u);   // eighth sign: even parity
            // one bit per byte, then a negated byte as (g ^ 0xFF) + 1: the magnitudes are 8, 25 or 43,
            // so the +1 never carries into the next byte
            const uint32_t nlo = ((s8 & 15u) * 0x00204081u) & 0x01010101u;
            const uint32_t nhi = ((s8 >> 4) * 0x00204081u) & 0x01010101u;
            w[2 * l] = (g.x ^ (nlo * 0xFFu)) + nlo;
            w[2 * l + 1] = (g.y ^ (nhi * 0xFFu)) + nhi;
        }
        const uint32_t w0[4] = {w[0], w[1], w[2], w[3]}, w1[4] = {w[4], w[5], w[6], w[7]};
        o.s[0] = dot4(w1, a.q[1]) + dot4(w0, a.q[0]);
        o.u[0] = dot4(w1, a.r[1]) + dot4(w0, a.r[0]);
        o.wsc[0] = h2f(lds16u(sb)) * (0.125f + 0.25f * float(ax.y >> 28));
        o.off[0] = 0.f;
    }
}

// sum-unit index (values sharing both scales: 16 for Q6_K, 32 otherwise) of scale group k of unit u
template <int FMT>
__device__ __forceinline__ int sum_unit(int u, int k) {
    if constexpr (FMT == F_Q4_0 || FMT == F_Q8_0 || FMT == F_IQ2_XXS || FMT == F_IQ4_XS || FMT == F_MXFP4 ||
                  FMT == F_IQ3_S || FMT == F_IQ3_XXS || FMT == F_Q4_1 || FMT == F_Q5_0 || FMT == F_Q5_1 ||
                  FMT == F_IQ4_NL || bits_format(FMT))
        return u;
    if constexpr (FMT == F_Q4_K || FMT == F_Q5_K) return 2 * u + k;   // unit u = sub-blocks 2u, 2u + 1 of the row
    if constexpr (FMT == F_Q3_K || iq2x_format(FMT) || FMT == F_Q2_K) return 2 * u + k;   // 16-value groups of unit u
    const int b = u >> 3, q = u & 7;
    if constexpr (FMT == F_Q6_K) {
        const int b6 = u >> 2, n = (u >> 1) & 1, h = u & 1;     // group k: values 128n + 32k + 16h.. of b6
        return b6 * 16 + 8 * n + 2 * k + h;
    }
    return b * 8 + 4 * (q >> 2) + k;    // TQ2_0
}

// the unit's contribution: sum over scale groups of wsc * (xd/254) * (254 S + S2) - off * xs
template <int FMT>
__device__ __forceinline__ float unit_dot(uint32_t rs, int u, const Act<FMT>& a, const uint2* grid) {
    UnitSums<FMT> o;
    unit_sums<FMT>(rs, u, a, o, grid);
    if constexpr (FMT == F_Q6_K) {
        // sum_g d sc_g * (xd_g / 254) * (254 S_g + S2_g), the codes' -32 folded into kk
        const int b = u >> 2, n = (u >> 1) & 1, h = u & 1;
        const uint32_t sb = rs + b * 210;
        uint32_t w[4][4];
        q6k_codes(sb, n, h, w);
        const float d = h2f(lds16u(sb + 208));
        float acc = 0.f;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const int4 x = a.q[g], y = a.r[g];
            const int s_ = dp4(w[g][1], x.y, dp4(w[g][0], x.x, 0)) + dp4(w[g][3], x.w, dp4(w[g][2], x.z, 0));
            const int t_ = dp4(w[g][1], y.y, dp4(w[g][0], y.x, 0)) + dp4(w[g][3], y.w, dp4(w[g][2], y.z, 0));
            const float wsc = d * float(int8_t(lds8u(sb + 192 + 8 * n + 2 * g + h)));
            acc = fmaf(wsc * a.d[g], float(254 * s_ + t_ - a.kk[g]), acc);
        }
        return acc;
    } else if constexpr (FMT == F_TQ2_0) {
        // d * (sum_g (xd_g / 254) (254 S_g + S2_g) - sum_g xs_g), codes c - 1 (quant.py:417-421): group g's
        // codes are bits 2g, 2g + 1 of each byte, masked in place (4^g times the code, exact in the int32
        // sums; a.d[g] carries the 4^-g)
        const int b = u >> 3, q = u & 7, n = q >> 2, j = q & 3;
        const uint32_t sb = rs + b * 66;
        const uint2 c = lds8_a2(sb + 32 * n + 8 * j);
        const float d = h2f(lds16u(sb + 64));
        const int xq[8] = {a.q[0].x, a.q[0].y, a.q[0].z, a.q[0].w, a.q[1].x, a.q[1].y, a.q[1].z, a.q[1].w};
        const int xr[8] = {a.r[0].x, a.r[0].y, a.r[0].z, a.r[0].w, a.r[1].x, a.r[1].y, a.r[1].z, a.r[1].w};
        float t = -a.s[0];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            const uint32_t m = 0x03030303u << (2 * g), c0 = c.x & m, c1 = c.y & m;
            const int s_ = dp4us(c1, xq[2 * g + 1], dp4us(c0, xq[2 * g], 0));
            const int u_ = dp4us(c1, xr[2 * g + 1], dp4us(c0, xr[2 * g], 0));
            t = fmaf(a.d[g], float(254 * s_ + u_), t);
        }
        return d * t;
    } else if constexpr (FMT == F_Q4_K || FMT == F_Q5_K) {
        // d * sum_k sc_k * (254 S_k + S2_k) * xd_k / 254  -  dmin * sum_k m_k * xs_k
        const float w = float(o.isc[0] * (254 * o.s[0] + o.u[0])) * a.d[0]
                      + float(o.isc[1] * (254 * o.s[1] + o.u[1])) * a.d[1];
        const float m = small_u2f(o.imn[0]) * a.s[0] + small_u2f(o.imn[1]) * a.s[1];
        return o.d * w - o.dm * m;
    } else {
        float acc = 0.f;
#pragma unroll
        for (int k = 0; k < UnitTraits<FMT>::NS; ++k)
            acc += o.wsc[k] * a.d[k] * float(254 * o.s[k] + o.u[k]) - o.off[k] * a.s[k];
        return acc;
    }
}

// ---- the kernel ---------------------------------------------------------------------------------

struct TileInfo {
    int slot, row0, nrows, job;
};

// The rows of all jobs / slots form one global row space; CTA c takes the contiguous range
// [c * total / grid, (c + 1) * total / grid) (equal bytes per CTA within one row) and walks it in
// tiles of at most R rows that never cross a job or slot boundary.
__device__ __forceinline__ long long cta_row_begin(const TmaParams& P, int c) {
    return (long long)c * P.total_rows / gridDim.x;
}

// the tile starting at global row g (< end of this CTA's range `hi`)
__device__ __forceinline__ TileInfo tile_at(const TmaParams& P, long long g, long long hi) {
    TileInfo t;
    long long start, stop;
    if (P.ids == nullptr) {
        int j = 0;
        while (j + 1 < P.n_jobs && g >= P.row_start[j + 1]) ++j;
        t.job = t.slot = j;
        start = P.row_start[j];
        stop = P.row_start[j + 1];
    } else {
        t.job = 0;
        t.slot = int(g / P.n_out[0]);
        start = (long long)t.slot * P.n_out[0];
        stop = start + P.n_out[0];
    }
    t.row0 = int(g - start);
    const long long lim = min(stop, hi);
    t.nrows = int(min((long long)P.rows_per_tile, lim - g));
    return t;
}

// weight base of a slot, or nullptr for an unused slot (id -1), a refused expert id or a misaligned
// table entry
__device__ __forceinline__ const uint8_t* tma_slot_base(const TmaParams& P, int slot) {
    if (P.ids == nullptr) return P.w[slot];
    const long long e = P.ids[slot];
    if (e < 0 || e >= P.n_exp) return nullptr;
    const uint8_t* base = P.per_expert >= 0 ? P.w[0] + e * P.per_expert
                                            : reinterpret_cast<const uint8_t*>(reinterpret_cast<const long long*>(P.w[0])[e]);
    return (reinterpret_cast<uintptr_t>(base) & 15u) ? nullptr : base;
}

// shared-memory layout: [stages x stage bytes][reduction 2 x NCW x R floats][codebook 2 KB]
//                      [fused activation: xq K, xq2 K, xd K/32, xs K/32 (XF only)][mbarriers]
#ifndef QMV_TMA_NPER                        // sweep builds may set another value
#define QMV_TMA_NPER 4
#endif
constexpr int kTmaRowsPerTeam = QMV_TMA_NPER;   // rows of a full tile per team (compile-time fast path)
// partial sums of rows spread over several warps: [row in window][warp in team], reduced once per window
constexpr int kPartFloats = 2048;
__host__ __device__ constexpr int tma_red_bytes(int ncw) { return kPartFloats * 4 + 0 * ncw; }
__host__ __device__ constexpr long long tma_act_bytes(int n_in) { return 2LL * n_in + n_in / 4; }
constexpr int kConsumerBarrier = 15;        // named barrier of all consumer warps (teams use 1..8)

// XF: 0 = the activation comes pre-quantised (P.xq ...), 1 = fp32 row in P.x, 2 = bf16 row in P.x,
// quantised by the CTA itself into shared memory (same arithmetic as quant_q8_kernel).
template <int FMT, int NCW, int G, int UPL, int XF, bool SUMS>
__global__ void __launch_bounds__(32 * (NCW + 1), NCW <= 8 ? 2 : 1) mv_tma_kernel(const TmaParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TEAMS = 32 * NCW / G;                  // rows processed side by side
    constexpr int WPT = G >= 32 ? G / 32 : 1;            // warps per team
    constexpr int NPER = kTmaRowsPerTeam;
    constexpr int VPU = UnitTraits<FMT>::VPU;
    const int R = P.rows_per_tile;
    const int S = P.stages;
    const long long stage_bytes = (long long)R * P.row_bytes;
    uint8_t* red_p = smem + S * stage_bytes;
    float* red = reinterpret_cast<float*>(red_p);
    uint2* grid = reinterpret_cast<uint2*>(red_p + tma_red_bytes(NCW));
    uint8_t* act_p = red_p + tma_red_bytes(NCW) + 2048;
    uint64_t* bars = reinterpret_cast<uint64_t*>(act_p + (XF ? tma_act_bytes(P.n_in) : 0));
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S);
    const uint32_t stage0 = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // the next kernel in the stream may start launching (its weight prefetch does not read our outputs)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, NCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if constexpr (FMT == F_IQ2_XXS) load_iq2xxs_grid(grid);
    if constexpr (FMT == F_IQ3_S) load_iq3s_grid(reinterpret_cast<uint32_t*>(grid));     // same 2 KB
    if constexpr (FMT == F_IQ3_XXS) load_iq3xxs_grid(reinterpret_cast<uint32_t*>(grid));
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer: weights only, no dependence on the previous kernel ----------------
        if (lane != 0) return;
        int it = 0, s = 0;                        // s = it % S, ph = (it / S) & 1, kept by increments
        uint32_t ph = 0;
        bool ok = true;
        const long long hi = cta_row_begin(P, blockIdx.x + 1);
        for (long long g = cta_row_begin(P, blockIdx.x); g < hi; ++it) {
            if (it >= S && !mbar_wait(empty0 + 8 * s, ph ^ 1)) {
                ok = false;
                break;
            }
            const TileInfo ti = tile_at(P, g, hi);
            g += ti.nrows;
            const uint8_t* base = tma_slot_base(P, ti.slot);
            if (base == nullptr) {
                // a refused id sets the status bit; an unused slot (id -1) is just zeros
                if (P.status && P.ids[ti.slot] != kPadSlot) atomicOr(P.status, DEV_BAD_ADDRESS);
                mbar_arrive(full0 + 8 * s);                   // nothing to copy: consumers write zeros
            } else {
                const uint32_t bytes = uint32_t((long long)ti.nrows * P.row_bytes);
                mbar_arrive_tx(full0 + 8 * s, bytes);
                bulk_g2s(stage0 + uint32_t(s * stage_bytes), base + (long long)ti.row0 * P.row_bytes, bytes,
                         full0 + 8 * s);
            }
            if (++s == S) {
                s = 0;
                ph ^= 1;
            }
        }
        if (!ok) {
            if (P.status) atomicOr(P.status, DEV_TIMEOUT);
            // drain: wait (bounded) for the copies of the last S iterations before leaving
            for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(full0 + 8 * (k % S), (k / S) & 1);
        }
        return;
    }

    // ---------------- consumers ----------------
    // Every consumer thread walks the same tiles and its team's named barriers, also after a timed-out
    // wait (then it only skips the work), so a failed wait can never leave a barrier short.
    const int cl = threadIdx.x;                 // 0 .. 32*NCW-1
    const int team = cl / G, li = cl % G;       // team (row slot), lane within the team
    const int U = P.n_in / VPU;                 // units per row
    // inputs written by the previous kernel are read only after it has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int8_t* sxq = nullptr;
    const int8_t* sxq2 = nullptr;
    const float* sxd = nullptr;
    const float* sxs = nullptr;
    if constexpr (XF != 0) {
        int8_t* wq = reinterpret_cast<int8_t*>(act_p);
        int8_t* wq2 = wq + P.n_in;
        float* wd = reinterpret_cast<float*>(wq2 + P.n_in);
        float* ws = wd + P.n_in / 32;
        const float* xf = static_cast<const float*>(P.x);
        const bool norm = XF == 1 && P.nw != nullptr;
        float inv = 1.f;
        if (norm) {
            // sum of v^2 in the norm kernel's order: 1024 threads, thread t over values t, t + 1024, ...,
            // a warp sum per warp of them, then one warp sum over the 32 warp sums (here every consumer
            // warp forms that last sum itself from shared memory; `red` is free until the first tile).
            // Warp w stands for norm-kernel warps w, w + NCW, ...; four rounds of loads in flight.
            constexpr int VPW = 32 / NCW;
            float ss[VPW];
#pragma unroll
            for (int j = 0; j < VPW; ++j) ss[j] = 0.f;
            for (int i0 = 0; i0 < P.n_in; i0 += 4 * 1024) {
                float v[VPW][4];
#pragma unroll
                for (int j = 0; j < VPW; ++j)
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int i = i0 + 1024 * k + 32 * (warp + NCW * j) + lane;
                        v[j][k] = i < P.n_in ? (P.nr ? __fadd_rn(xf[i], __fmul_rn(P.nrs, P.nr[i])) : xf[i]) : 0.f;
                    }
#pragma unroll
                for (int j = 0; j < VPW; ++j)
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (i0 + 1024 * k + 32 * (warp + NCW * j) + lane < P.n_in) ss[j] = __fmaf_rn(v[j][k], v[j][k], ss[j]);
            }
#pragma unroll
            for (int j = 0; j < VPW; ++j) {
                const float t = warp_sum(ss[j]);
                if (lane == 0) red[warp + NCW * j] = t;
            }
            named_sync(kConsumerBarrier, 32 * NCW);
            inv = rsqrtf(warp_sum(red[lane]) / float(P.n_in) + P.neps);
        }
        // a group on each eighth of a warp, QB rounds of a warp's loads in flight before their groups
        constexpr int QB = 4;
        const int n_grp = P.n_in / 32;
        const int eighth = lane >> 3, m = lane & 7;
        for (int g0 = warp * 4 * QB; g0 < n_grp; g0 += NCW * 4 * QB) {
            float v[QB][4];
#pragma unroll
            for (int b = 0; b < QB; ++b) {
                const int grp = min(g0 + 4 * b + eighth, n_grp - 1);      // past the end: a copy, not stored
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int i = 32 * grp + m + 8 * k;
                    if (XF == 1 && norm) {
                        const float h = P.nr ? __fadd_rn(xf[i], __fmul_rn(P.nrs, P.nr[i])) : xf[i];
                        v[b][k] = __fmul_rn(__fmul_rn(h, inv), P.nw[i]);
                    } else {
                        v[b][k] = XF == 1 ? xf[i] : bf2f(static_cast<const uint16_t*>(P.x)[i]);
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < QB; ++b) {
                const int grp = g0 + 4 * b + eighth;
                quantize_group8(v[b], 32LL * grp, grp < n_grp, wq, wq2, wd, ws);
            }
        }
        if (norm && P.nr && P.nh) {
            // v = h + rs r back to memory, a slice per CTA (no store among the loads above: a store there
            // would keep the compiler from batching them)
            const int lo = int((long long)blockIdx.x * P.n_in / gridDim.x);
            const int hi = int((long long)(blockIdx.x + 1) * P.n_in / gridDim.x);
            for (int i = lo + int(threadIdx.x); i < hi; i += 32 * NCW)
                P.nh[i] = __fadd_rn(xf[i], __fmul_rn(P.nrs, P.nr[i]));
        }
        named_sync(kConsumerBarrier, 32 * NCW);
        sxq = wq; sxq2 = wq2; sxd = wd; sxs = ws;
    }
    Act<FMT> act[UPL];
    long long cur_row = -1;
    bool dead = false;
    int it = 0, s = 0;                          // s = it % S, ph = (it / S) & 1
    uint32_t ph = 0;
    // window of rows whose cross-warp partial sums wait in shared memory (teams wider than a warp)
    constexpr int PR = kPartFloats / WPT;
    float* part = red;
    int w_job = 0, w_row0 = 0, w_rows = 0;
    auto flush = [&]() {                                    // every consumer thread, uniformly
        named_sync(kConsumerBarrier, 32 * NCW);
        if (!dead) {
            float* y = P.ids == nullptr ? P.y[w_job] : P.y[0] + (long long)w_job * P.n_out[0];
            for (int rl = cl; rl < w_rows; rl += 32 * NCW) {
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < WPT; ++w) v += part[rl * WPT + w];
                y[w_row0 + rl] = v;
            }
        }
        named_sync(kConsumerBarrier, 32 * NCW);
        if (!dead && P.ids == nullptr) ep_groups(P, w_job, w_row0, w_rows, warp, NCW);
        w_rows = 0;
    };
    const long long hi = cta_row_begin(P, blockIdx.x + 1);
    for (long long g = cta_row_begin(P, blockIdx.x); g < hi; ++it) {
        const TileInfo ti = tile_at(P, g, hi);
        g += ti.nrows;
        const long long arow = P.ids == nullptr ? 0 : ti.slot / P.x_group;
        if (arow != cur_row) {
            const long long off = arow * P.n_in;
#pragma unroll
            for (int i = 0; i < UPL; ++i) {
                const int u = li + G * i;
                if (u < U) {
                    if constexpr (XF != 0) load_act<FMT, true, SRC_SMEM>(act[i], u, sxq, sxq2, sxd, sxs);
                    else load_act<FMT, !SUMS>(act[i], u, P.xq + off, P.xq2 + off, P.xd + off / 32, P.xs + off / 32);
                }
            }
            cur_row = arow;
        }
        const bool got = !dead && mbar_wait(full0 + 8 * s, ph);
        if (!got && !dead) {
            dead = true;
            if (lane == 0 && P.status) atomicOr(P.status, DEV_TIMEOUT);
        }
        const bool work = got && !(P.ids != nullptr && tma_slot_base(P, ti.slot) == nullptr);
        const uint32_t st = stage0 + uint32_t(s * stage_bytes);
        float acc[NPER];
#pragma unroll
        for (int i = 0; i < NPER; ++i) acc[i] = 0.f;
        if (work && 4 * ti.nrows >= 3 * R && R == NPER * TEAMS && !SUMS) {
            // a full tile, or one at least 3/4 full (a 4096-row matrix's 27-28 rows a CTA): NPER
            // independent rows per lane, no per-row guards (the compiler interleaves them); a short
            // tile's rows past nrows compute on what the stage holds there (inside the stage; the
            // stores below are guarded)
#pragma unroll
            for (int k = 0; k < UPL; ++k) {
                const int u = li + G * k;
                if (u < U) {
#pragma unroll
                    for (int i = 0; i < NPER; ++i)
                        acc[i] += unit_dot<FMT>(st + uint32_t((team + TEAMS * i) * P.row_bytes), u, act[k], grid);
                }
            }
        } else if (work) {
#pragma unroll
            for (int i = 0; i < NPER; ++i) {
                const int r = team + TEAMS * i;
                if (r < ti.nrows) {
                    const uint32_t rs = st + uint32_t(r * P.row_bytes);
#pragma unroll
                    for (int k = 0; k < UPL; ++k) {
                        const int u = li + G * k;
                        if (u < U) {
                            if constexpr (SUMS) {
                                UnitSums<FMT> o;
                                unit_sums<FMT>(rs, u, act[k], o, grid);
                                const long long row = ti.row0 + r;
                                const int upr = P.n_in / unit_values(FMT);
#pragma unroll
                                for (int q = 0; q < UnitTraits<FMT>::NS; ++q) {
                                    atomicAdd(P.s + row * upr + sum_unit<FMT>(u, q), o.s[q]);
                                    atomicAdd(P.s2 + row * upr + sum_unit<FMT>(u, q), o.u[q]);
                                }
                            } else {
                                acc[i] += unit_dot<FMT>(rs, u, act[k], grid);
                            }
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (got && lane == 0) mbar_arrive(empty0 + 8 * s);   // this warp is done with the stage
        if (++s == S) {
            s = 0;
            ph ^= 1;
        }
        if constexpr (!SUMS) {
            if constexpr (G <= 32) {
                float* y = P.ids == nullptr ? P.y[ti.job] : P.y[0] + (long long)ti.slot * P.n_out[0];
#pragma unroll
                for (int i = 0; i < NPER; ++i) {
                    float v = acc[i];
#pragma unroll
                    for (int o = G / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    const int r = team + TEAMS * i;
                    if (li == 0 && got && r < ti.nrows) y[ti.row0 + r] = v;
                }
            } else {
                const int wjob = P.ids == nullptr ? ti.job : ti.slot;
                if (w_rows > 0 && (wjob != w_job || ti.row0 != w_row0 + w_rows || w_rows + ti.nrows > PR)) flush();
                if (w_rows == 0) {
                    w_job = wjob;
                    w_row0 = ti.row0;
                }
                const int wt = li >> 5;                      // warp within the team
#pragma unroll
                for (int i = 0; i < NPER; ++i) {
                    const float v = warp_sum(acc[i]);
                    const int r = team + TEAMS * i;
                    if (lane == 0 && r < ti.nrows) part[(w_rows + r) * WPT + wt] = v;
                }
                w_rows += ti.nrows;
            }
        }
    }
    if constexpr (!SUMS && G > 32) {
        if (w_rows > 0) flush();
    }
}

}  // namespace qmv
