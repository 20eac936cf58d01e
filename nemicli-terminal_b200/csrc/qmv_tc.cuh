// Tensor-core tile path for 16..128 tokens (the reference's MMQ, ggufengine/mmvq.py:536-724, dispatched
// for MMVQ_BIS < M <= MMQ_BIS at models/common.py:406-407), on the 5th-generation tensor cores.
//
//   y[t][r] = xs[t] * sum_k f16(W[r, k]) * f16(x[t, k] / xs[t]),   xs[t] = max_k |x[t, k]| / 256
//
// The arithmetic is the reference's: every weight value is unpacked to fp16 from its fp32 form
// (Q4_K: d sc q - dmin m as one fused multiply-add; Q6_K: d sc (q - 32)), every token scaled to
// |x| <= 256 in fp16, products summed in fp32.  What differs is the machine:
//
//   CTA tile    128 weight rows (the MMA's M) x N tokens (N = tokens rounded up to 16, at most 128), one
//               fp32 accumulator of 128 lanes x N columns in tensor memory;
//   K steps     64 values (shared memory 2 x (16 KB + N x 128 B): three or four CTAs an SM): each of the 128 threads unpacks its row's 64 values (loaded one step ahead in
//               registers) into shared memory in the canonical K-major layout without swizzle (core
//               matrices of 8 rows x 16 bytes, 128 B apart along K, 1 KB apart per 8 rows), copies the
//               tokens' 64 fp16 values the same way, and one thread issues four kind::f16 MMAs
//               (K = 16 each) and commits them to the stage's mbarrier; two stages alternate, so the
//               tensor cores work on step k while the threads unpack step k + 1;
//   split-K     the row tiles x K parts fill the SMs; each part's scaled sums go to a workspace and the
//               last part of a tile to finish (a counter per tile) adds the parts in part order, so the
//               result does not depend on timing (the reference adds its parts with atomics).
//
// Every mbarrier wait is bounded; on expiry the CTA sets QMV_DEV_TIMEOUT, waits (bounded) for its
// MMAs, frees its tensor memory and leaves.
#pragma once
#include <cuda_fp16.h>

#include "qmv_tma.cuh"

namespace qmv {

constexpr int kTcRows = 128;               // weight rows per CTA tile (MMA M)
constexpr int kTcK = 64;                   // K values per step
constexpr int kTcMaxN = 128;               // tokens per launch
constexpr int kTcThreads = 256;            // two threads per weight row
constexpr int kTcStageA = kTcRows * kTcK * 2;    // 16 KB
constexpr int kTcStageB = kTcMaxN * kTcK * 2;    // 16 KB
constexpr int kTcSmem = 2 * (kTcStageA + kTcStageB) + 64;    // at N = 128; a launch takes 2 (A + N 128 B) + 64
__host__ __device__ constexpr int tc_smem(int n_pad) { return 2 * (kTcStageA + n_pad * kTcK * 2) + 64; }
constexpr float kTcScale = 256.0f;         // tokens scaled to |x| <= 256 (the reference's MMQ_SKALA)

struct TcParams {
    const uint8_t* w;          // n_out rows of row_bytes
    long long row_bytes;
    int n_out, n_in;
    const uint16_t* xh;        // [n_tok][n_in] fp16, x / xs
    const float* xs;           // [n_tok]
    int n_tok, n_pad;          // tokens, and the MMA's N (multiple of 16)
    int splits;                // K parts
    float* part;               // [splits][n_tok][n_out] scaled sums (splits > 1)
    int* done;                 // per row tile: parts finished (zeroed by the input kernel)
    float* y;                  // [n_tok][n_out]
    int* status;
};

// ---- tcgen05 wrappers -------------------------------------------------------------------------

// shared-memory matrix descriptor, K-major without swizzle: start, leading (K) and stride (8-row)
// byte offsets, descriptor version 1 (bits 46-47)
__device__ __forceinline__ uint64_t tc_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t((lbo >> 4) & 0x3FFFu) << 16) |
           (uint64_t((sbo >> 4) & 0x3FFFu) << 32) | (uint64_t(1) << 46);
}
// instruction descriptor of kind::f16: fp32 accumulator, fp16 A and B, both K-major, M = 128, N
__host__ __device__ constexpr uint32_t tc_idesc(int n) {
    return (1u << 4) | (0u << 7) | (0u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(kTcRows >> 4) << 24);
}
__device__ __forceinline__ void tc_mma(uint32_t tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
                 :: "r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// 8 consecutive fp32 columns of the warp's 32 lanes (one lane = one row) from tensor memory
__device__ __forceinline__ void tc_ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ uint32_t f2h2(float lo, float hi) {    // two fp32 -> fp16x2, round to nearest
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

// ---- input: one CTA per token (the reference's mmq_eingang, ggufengine/mmvq.py:604-632) ----------

// xs = max(max|x|, 1e-30) / 256, xh = fp16(x * (1 / xs)); CTA 0 also zeroes the tile counters
__global__ void __launch_bounds__(256) tc_input_kernel(const void* __restrict__ x, int x_f32, int n,
                                                       uint16_t* __restrict__ xh, float* __restrict__ xs,
                                                       int* __restrict__ done, int n_done) {
    __shared__ float red[8];
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < n_done; i += blockDim.x) done[i] = 0;
    const long long z = (long long)blockIdx.x * n;
    float m = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x_f32 ? static_cast<const float*>(x)[z + i] : bf2f(static_cast<const uint16_t*>(x)[z + i]);
        m = fmaxf(m, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
        m = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (threadIdx.x == 0) red[0] = __fdiv_rn(fmaxf(m, 1e-30f), kTcScale);
    }
    __syncthreads();
    const float s = red[0], inv = __fdiv_rn(1.0f, s);
    if (threadIdx.x == 0) xs[blockIdx.x] = s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = x_f32 ? static_cast<const float*>(x)[z + i] : bf2f(static_cast<const uint16_t*>(x)[z + i]);
        xh[z + i] = __half_as_ushort(__float2half_rn(__fmul_rn(v, inv)));
    }
}

// ---- one thread's row of a K step: raw bytes (loaded a step ahead), then 64 fp16 values --------

template <int FMT> struct TcRaw;
// Thread half hf of a row takes k-cores 2 hf, 2 hf + 1 of each 32-value half of the step (values
// 16 hf .. 16 hf + 15 of each).
// Q4_K: the 16-byte header and qs bytes 32 p + 16 hf .. + 15 (their low nibbles: sub-block 2p, high: 2p + 1)
template <> struct TcRaw<F_Q4_K> {
    uint4 hd, q;
    __device__ __forceinline__ void load(const uint8_t* row, int c, int hf) {
        const uint8_t* sb = row + (c >> 2) * 144;
        hd = ldw16(sb);
        q = ldw16(sb + 16 + 32 * (c & 3) + 16 * hf);
    }
};
// Q6_K: for half n = (c >> 1) & 1 of superblock c >> 2 (groups 2 (c & 1), 2 (c & 1) + 1): ql bytes
// 64 n + 16 hf .. and 64 n + 32 + 16 hf .. (16 each), qh bytes 32 n + 16 hf .., the half's 8 int8 scales
// and d (2-byte aligned superblocks); the same bytes serve steps c and c ^ 1
template <> struct TcRaw<F_Q6_K> {
    uint4 la, lb, hq;
    uint2 sc;
    uint32_t d;
    __device__ __forceinline__ void load(const uint8_t* row, int c, int hf) {
        const uint8_t* sb = row + (c >> 2) * 210;
        const int n = (c >> 1) & 1;
        la = ldw16_a2(sb + 64 * n + 16 * hf);
        lb = ldw16_a2(sb + 64 * n + 32 + 16 * hf);
        hq = ldw16_a2(sb + 128 + 32 * n + 16 * hf);
        sc = ldw8_a2(sb + 192 + 8 * n);
        d = ldw2(sb + 208);
    }
};

// Q6_K: scale of (group G, half l / 16) = int8 byte l / 16 + 2 G of the half's 8
__device__ __forceinline__ float tc_scale_q6k(const TcRaw<F_Q6_K>& r, int G, int half16) {
    const int i = half16 + 2 * G;
    const uint32_t w = i < 4 ? r.sc.x : r.sc.y;
    const int s = int(int8_t((w >> (8 * (i & 3))) & 0xFFu));
    return __fmul_rn(h2f(r.d), float(s));
}

// the 8 values of k-core kc (k = 8 kc .. 8 kc + 7 of the step) as four fp16x2 words
template <int FMT>
__device__ __forceinline__ uint4 tc_unpack(const TcRaw<FMT>& r, int c, int kc, const float (&a)[2], const float (&b)[2]);

// reference schreib_q4k (ggufengine/mmvq.py:578-592): value = fp16(d sc q - dmin m), d sc and dmin m in fp32,
// one fused multiply-add
template <>
__device__ __forceinline__ uint4 tc_unpack<F_Q4_K>(const TcRaw<F_Q4_K>& r, int, int kc, const float (&a)[2],
                                                   const float (&b)[2]) {
    const int g = kc >> 2;                              // 0: sub-block 2p (low nibbles), 1: 2p + 1 (high)
    const int w = 2 * (kc & 1);                         // the thread's qs words w, w + 1 (bytes 8 (kc & 3) ..)
    const uint32_t W[4] = {r.q.x, r.q.y, r.q.z, r.q.w};
    const uint32_t sh = 4u * uint32_t(g);
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t v = W[w + i] >> sh;
        const float f0 = __fmaf_rn(a[g], small_u2f(v & 15u), -b[g]);
        const float f1 = __fmaf_rn(a[g], small_u2f((v >> 8) & 15u), -b[g]);
        const float f2 = __fmaf_rn(a[g], small_u2f((v >> 16) & 15u), -b[g]);
        const float f3 = __fmaf_rn(a[g], small_u2f((v >> 24) & 15u), -b[g]);
        o[2 * i] = f2h2(f0, f1);
        o[2 * i + 1] = f2h2(f2, f3);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// reference schreib_q6k (ggufengine/mmvq.py:606-616): value = fp16(d sc (q - 32)), d sc in fp32.  Step
// values 0..31 are group 2h (32 k-values of the half), 32..63 group 2h + 1; value l of group G takes ql
// byte 64n + l + 32 (G & 1) (low nibble for G < 2, high for G >= 2) and qh bits 2G.. of byte 32n + l,
// scale sc[l / 16 + 2 G]
template <>
__device__ __forceinline__ uint4 tc_unpack<F_Q6_K>(const TcRaw<F_Q6_K>& r, int c, int kc, const float (&)[2],
                                                   const float (&)[2]) {
    const int hsel = c & 1, j = kc >> 2, G = 2 * hsel + j;
    const int l0 = 8 * (kc & 3);                         // first l of the k-core (16 hf or 16 hf + 8)
    const int lw0 = 2 * (kc & 1);                        // its words in the thread's 16-byte runs
    const uint4 lsel = j ? r.lb : r.la;
    const uint32_t L[4] = {lsel.x, lsel.y, lsel.z, lsel.w};
    const uint32_t H[4] = {r.hq.x, r.hq.y, r.hq.z, r.hq.w};
    const float f = tc_scale_q6k(r, G, l0 >> 4);         // d * sc[l / 16 + 2 G]
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t lw = L[lw0 + i] >> (G >= 2 ? 4 : 0);
        const uint32_t hw = H[lw0 + i] >> (2 * G);
        const uint32_t q = (lw & 0x0F0F0F0Fu) | ((hw & 0x03030303u) << 4);
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = __fmul_rn(f, float(int((q >> (8 * e)) & 63u) - 32));
        o[2 * i] = f2h2(v[0], v[1]);
        o[2 * i + 1] = f2h2(v[2], v[3]);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// per-step scales of Q4_K: a = d sc, b = dmin m of the two sub-blocks (Q6_K takes its scale per k-core)
__device__ __forceinline__ void tc_scales(const TcRaw<F_Q4_K>& r, int c, float (&a)[2], float (&b)[2]) {
    int isc[2];
    uint32_t imn[2];
    kquant_scales(r.hd, c & 3, isc, imn);
    const float d = h2f(r.hd.x & 0xFFFFu), dm = h2f(r.hd.x >> 16);
    a[0] = __fmul_rn(d, float(isc[0]));
    a[1] = __fmul_rn(d, float(isc[1]));
    b[0] = __fmul_rn(dm, float(imn[0]));
    b[1] = __fmul_rn(dm, float(imn[1]));
}

__device__ __forceinline__ void tc_scales(const TcRaw<F_Q6_K>&, int, float (&a)[2], float (&b)[2]) {
    a[0] = a[1] = b[0] = b[1] = 0.f;
}

__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" :: "r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

// ---- the kernel: CTA = (row tile, K part); thread t = row t of the tile while unpacking, rows 32 w .. of
// warp w while reading the accumulator back -------------------------------------------------------

template <int FMT>
__global__ void __launch_bounds__(kTcThreads) tc_mm_kernel(const TcParams P) {
    extern __shared__ __align__(1024) uint8_t tc_smem[];
    __shared__ int s_last;
    const uint32_t base = smem_u32(tc_smem);
    const uint32_t sa[2] = {base, base + uint32_t(kTcStageA)};
    const uint32_t bst = uint32_t(P.n_pad * kTcK * 2);                        // B stage: N rows of 128 B
    const uint32_t sb[2] = {base + uint32_t(2 * kTcStageA), base + uint32_t(2 * kTcStageA) + bst};
    const uint32_t bar0 = base + uint32_t(2 * kTcStageA) + 2 * bst;           // two mbarriers, 8 B each
    uint32_t* tslot = reinterpret_cast<uint32_t*>(tc_smem + 2 * kTcStageA + 2 * bst + 16);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x / P.splits, part = blockIdx.x % P.splits;
    const int chunks = P.n_in / kTcK;
    const int c0 = int((long long)part * chunks / P.splits), c1 = int((long long)(part + 1) * chunks / P.splits);
    const int rr = tid >> 1, hf = tid & 1;                 // this thread's row of the tile and its half
    const int row = tile * kTcRows + rr;
    const uint8_t* wrow = P.w + (long long)min(row, P.n_out - 1) * P.row_bytes;   // rows past the end: discarded
    const uint32_t cols = P.n_pad <= 32 ? 32u : P.n_pad <= 64 ? 64u : 128u;
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" :: "r"(smem_u32(tslot)), "r"(cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(bar0, 1);
        mbar_init(bar0 + 8, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tslot;
    const uint32_t idesc = tc_idesc(P.n_pad);
    // token values: 16-byte pieces (one core-matrix row), n_pad * 8 per step; thread t takes t + 128 i
    constexpr int kBPer = kTcMaxN * 8 / kTcThreads;
    TcRaw<FMT> raw, raw_next;                            // step c, and step c + 1 (loaded a step earlier)
    uint4 xb[kBPer];
    auto load_x = [&](int c) {
#pragma unroll
        for (int i = 0; i < kBPer; ++i) {
            const int j = tid + kTcThreads * i, n = j >> 3, kc = j & 7;
            xb[i] = n < P.n_tok ? __ldg(reinterpret_cast<const uint4*>(P.xh + (long long)n * P.n_in + c * kTcK + 8 * kc))
                                : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    bool dead = false;
    int issued = c0;                                     // steps whose MMAs were issued: [c0, issued)
    if (c0 < c1) {
        raw.load(wrow, c0, hf);
        load_x(c0);
    }
    // a Q6_K half serves two steps (c even, c + 1): the odd step reuses the even one's bytes
    auto next_of = [&](int c) {
        if (FMT == F_Q6_K && (c & 1)) raw_next = raw;
        else raw_next.load(wrow, c, hf);
    };
    if (c0 + 1 < c1) next_of(c0 + 1);
    for (int c = c0; c < c1; ++c) {
        const int s = (c - c0) & 1, use = (c - c0) >> 1;
        // stage s was last read by the MMAs of step c - 2 (the stage's use - 1 th commit)
        const bool ok = c - c0 < 2 || mbar_wait(bar0 + 8 * s, uint32_t(use - 1) & 1u);
        float a[2], b[2];
        tc_scales(raw, c, a, b);
        const uint32_t arow = sa[s] + uint32_t((rr >> 3) * 1024 + (rr & 7) * 16);
#pragma unroll
        for (int i = 0; i < 4; ++i) {                       // k-cores 2 hf, 2 hf + 1, 4 + 2 hf, 5 + 2 hf
            const int kc = (i >> 1) * 4 + 2 * hf + (i & 1);
            sts128(arow + kc * 128, tc_unpack<FMT>(raw, c, kc, a, b));
        }
#pragma unroll
        for (int i = 0; i < kBPer; ++i) {
            const int j = tid + kTcThreads * i, n = j >> 3, kc = j & 7;
            if (n < P.n_pad) sts128(sb[s] + uint32_t((n >> 3) * 1024 + kc * 128 + (n & 7) * 16), xb[i]);
        }
        // weights two steps ahead, token values one
        raw = raw_next;
        if (c + 2 < c1) next_of(c + 2);
        if (c + 1 < c1) load_x(c + 1);
        fence_async_smem();                              // the generic-proxy stores, before the MMAs read them
        tc_fence_before();
        const int fail = __syncthreads_or(!ok);
        tc_fence_after();
        if (fail) {
            dead = true;
            break;
        }
        if (tid == 0) {
#pragma unroll
            for (int kk = 0; kk < kTcK / 16; ++kk)
                tc_mma(tmem, tc_desc(sa[s] + kk * 256, 128, 1024), tc_desc(sb[s] + kk * 256, 128, 1024), idesc,
                       (c > c0 || kk > 0) ? 1u : 0u);
            tc_commit(bar0 + 8 * s);
        }
        issued = c + 1;
    }
    // the last commit covers every MMA the CTA issued
    bool ok = true;
    if (issued > c0) {
        const int L = issued - 1 - c0;
        ok = mbar_wait(bar0 + 8 * (L & 1), uint32_t(L >> 1) & 1u);
    }
    const int fail = __syncthreads_or(!ok);
    tc_fence_after();
    if (dead || fail || issued == c0) {
        if (tid == 0 && P.status) atomicOr(P.status, DEV_TIMEOUT);
    } else {
        // warp w reads lanes 32 (w & 3) .. (its quadrant) and the columns of half w >> 2
        const int quad = warp & 3, half_cols = P.n_pad / 2;
        const int r = tile * kTcRows + 32 * quad + lane;
        float* dst = P.splits > 1 ? P.part + (long long)part * P.n_tok * P.n_out : P.y;
        for (int col = (warp >> 2) * half_cols; col < (warp >> 2) * half_cols + half_cols; col += 8) {
            float v[8];
            tc_ld8(tmem + (uint32_t(32 * quad) << 16) + uint32_t(col), v);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int t = col + j;
                if (t < P.n_tok && r < P.n_out) dst[(long long)t * P.n_out + r] = __fmul_rn(v[j], __ldg(P.xs + t));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(tmem), "r"(cols) : "memory");
    if (P.splits > 1) {
        // the tile's last part adds the parts in part order
        __threadfence();
        __syncthreads();
        if (tid == 0) s_last = atomicAdd(P.done + tile, 1) == P.splits - 1;
        __syncthreads();
        if (s_last) {
            __threadfence();
            // row per thread (two threads a row: alternate blocks of 8 tokens), 8 independent loads per
            // part in flight
            const int r = tile * kTcRows + (tid & (kTcRows - 1));
            if (r < P.n_out) {
                for (int t0 = 8 * (tid / kTcRows); t0 < P.n_tok; t0 += 8 * (kTcThreads / kTcRows)) {
                    float v[8];
#pragma unroll
                    for (int j = 0; j < 8; ++j) v[j] = 0.f;
                    for (int q = 0; q < P.splits; ++q) {
                        const float* src = P.part + ((long long)q * P.n_tok + t0) * P.n_out + r;
                        float u[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) u[j] = t0 + j < P.n_tok ? __ldcg(src + (long long)j * P.n_out) : 0.f;
#pragma unroll
                        for (int j = 0; j < 8; ++j) v[j] = __fadd_rn(v[j], u[j]);
                    }
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        if (t0 + j < P.n_tok) P.y[(long long)(t0 + j) * P.n_out + r] = v[j];
                }
            }
        }
    }
}

}  // namespace qmv
