// Kernels of the quantized matvec path: activation quantisation and the per-format int8 matvec.
//
// Activation input ("Eingang", the reference's name; ggufengine/mmvq.py:825-849): per 32 values
// an int8 xq with scale xd = amax/127, a second int8 xq2 holding the remainder at scale xd/254,
// and xs = the fp32 sum of the 32 values.  The matvec computes, per 32-value group g of a row,
//     y += wscale * xd_g * (S + S2/254) - offs * xs_g,   S = sum code*xq, S2 = sum code*xq2 (int32)
// with the per-format weight code, weight scale and offset of ggufengine/quant.py.
#pragma once
#include "qmv_common.cuh"

namespace qmv {

// ---------------------------------------------------------------------------------------------
// Activation quantisation (restates ggufengine/mmvq.py:59-83 with IEEE-rounded division)
// ---------------------------------------------------------------------------------------------

// One warp quantises one group of 32 consecutive values; lane l holds value l of the group.
__device__ __forceinline__ void quantize_group(float v, long long i, int8_t* __restrict__ xq,
                                               int8_t* __restrict__ xq2, float* __restrict__ xd,
                                               float* __restrict__ xs) {
    float a = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
    const float d = __fdiv_rn(a, 127.0f);
    const float d2 = __fdiv_rn(d, 254.0f);
    int q = 0, q2 = 0;
    if (d > 0.f) {
        q = __float2int_rn(__fdiv_rn(v, d));
        const float r = __fmaf_rn(-float(q), d, v);
        q2 = max(-127, min(127, __float2int_rn(__fdiv_rn(r, d2))));
    }
    const float s = warp_sum(v);          // butterfly xor 16..1: the order the oracle restates
    xq[i] = int8_t(q);
    xq2[i] = int8_t(q2);
    if ((threadIdx.x & 31) == 0) {
        xd[i >> 5] = d;
        xs[i >> 5] = s;
    }
}

// One group of 32 values on 8 lanes (an aligned eighth of a warp): lane m holds values m, m+8, m+16
// and m+24 of the group starting at value i0 in v[0..3].  The arithmetic of quantize_group: the group
// maximum in any order (exact), and the fp32 sum in the butterfly order of warp_sum as lane 0 forms it,
// (v_m + v_m+16) + (v_m+8 + v_m+24) in the lane, then xor 4, 2, 1 across the eight lanes.  Stores only
// if `store` (the shuffles run in every lane).
__device__ __forceinline__ void quantize_group8(const float (&v)[4], long long i0, bool store,
                                                int8_t* __restrict__ xq, int8_t* __restrict__ xq2,
                                                float* __restrict__ xd, float* __restrict__ xs) {
    float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
    float s = (v[0] + v[2]) + (v[1] + v[3]);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
        s += __shfl_xor_sync(0xffffffffu, s, o);
    }
    const float d = __fdiv_rn(a, 127.0f);
    const float d2 = __fdiv_rn(d, 254.0f);
    const int m = threadIdx.x & 7;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        int q = 0, q2 = 0;
        if (d > 0.f) {
            q = __float2int_rn(__fdiv_rn(v[k], d));
            const float r = __fmaf_rn(-float(q), d, v[k]);
            q2 = max(-127, min(127, __float2int_rn(__fdiv_rn(r, d2))));
        }
        if (store) {
            xq[i0 + m + 8 * k] = int8_t(q);
            xq2[i0 + m + 8 * k] = int8_t(q2);
        }
    }
    if (store && m == 0) {
        xd[i0 >> 5] = d;
        xs[i0 >> 5] = s;
    }
}

// the gated activation of act_q8 (ggufengine/mmvq.py:120-131): SiLU, or GELU in its tanh form, of x,
// times u (has_u); one definition for the producer kernel and the staged matvec's epilogue
__device__ __forceinline__ float act_value(float x, float u, bool has_u, int gelu) {
    float v = gelu ? 0.5f * x * (1.f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x))) : x / (1.f + expf(-x));
    if (has_u) v *= u;
    return v;
}

static __global__ void __launch_bounds__(256) quant_q8_kernel(const void* __restrict__ x, int x_f32,
                                                       int8_t* __restrict__ xq, int8_t* __restrict__ xq2,
                                                       float* __restrict__ xd, float* __restrict__ xs,
                                                       long long n) {
    // with programmatic dependent launch: the next kernel may launch now; nothing is read or written
    // before the previous kernel has completed
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if ((i & ~31LL) >= n) return;          // n % 32 == 0: whole warps leave together
    const float v = x_f32 ? static_cast<const float*>(x)[i] : bf2f(static_cast<const uint16_t*>(x)[i]);
    quantize_group(v, i, xq, xq2, xd, xs);
}

// ---------------------------------------------------------------------------------------------
// Matvec
// ---------------------------------------------------------------------------------------------

struct MvParams {
    const uint8_t* w;          // weights; with ids: the expert tensor, or (per_expert < 0) an int64 address table
    const long long* ids;      // expert id per slot, or nullptr (one slot: w itself)
    long long per_expert;      // bytes per expert (>= 0), or -1: w is an address table
    long long row_bytes;       // bytes per weight row
    const int8_t* xq;
    const int8_t* xq2;
    const float* xd;
    const float* xs;
    int x_group;               // slots per activation row: slot j reads row j / x_group (rows n_in values apart)
    float* y;                  // [slot][token][n_out]
    int32_t* s;                // sums mode: [row][unit] int32 sums of code*xq
    int32_t* s2;               //            ... and of code*xq2
    int* status;               // device status word (bits DEV_*)
    long long n_exp;           // experts addressable through ids (ids outside [0, n_exp) are refused)
    int n_out, n_in, slots;
};

// Per-lane work: a warp walks a row group of RW rows; lane = 8 * (superblock % 4) + q, where the
// 8 lanes of a 256-value superblock split it into eight 32-value pieces (per format below).
// tb[t]: activation value offset of token t's row start.  acc[r][t]: partial dot products.

template <int T>
struct Tok {
    long long tb[T];
};

// ---- Q4_K: 144 B = d, dmin (f16), 12 B of 6-bit scales/mins, 128 B nibbles (quant.py:111-120).
// Lane q takes qs bytes 16q..16q+15: the low nibbles are values 16h..16h+15 of sub-block 2p, the
// high nibbles the same values of sub-block 2p+1 (p = q/2, h = q%2).
// Q5_K (Q5 = true): 176 B = the same header, qh[32] at 16, qs[128] at 48 (quant.py:123-137); bit 2p
// (low nibbles) or 2p+1 (high nibbles) of qh[16h + i] is bit 4 of the code, unsigned 0..31.
template <int T, int RW, bool SUMS, bool Q5 = false>
__device__ __forceinline__ void lane_q4k(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int p = q >> 1, h = q & 1;
    uint32_t lo[RW][4], hi[RW][4];
    float d[RW], dm[RW], sc0[RW], sc1[RW], m0[RW], m1[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * (Q5 ? 176 : 144);
        const uint4 hd = ldw16(b);
        const uint4 v = ldw16(b + (Q5 ? 48 : 16) + 16 * q);
        lo[r][0] = v.x & 0x0F0F0F0Fu; hi[r][0] = (v.x >> 4) & 0x0F0F0F0Fu;
        lo[r][1] = v.y & 0x0F0F0F0Fu; hi[r][1] = (v.y >> 4) & 0x0F0F0F0Fu;
        lo[r][2] = v.z & 0x0F0F0F0Fu; hi[r][2] = (v.z >> 4) & 0x0F0F0F0Fu;
        lo[r][3] = v.w & 0x0F0F0F0Fu; hi[r][3] = (v.w >> 4) & 0x0F0F0F0Fu;
        if constexpr (Q5) {
            const uint4 qh = ldw16(b + 16 + 16 * h);
            const uint32_t H[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo[r][i] |= ((H[i] >> (2 * p)) & 0x01010101u) << 4;
                hi[r][i] |= ((H[i] >> (2 * p + 1)) & 0x01010101u) << 4;
            }
        }
        d[r] = h2f(hd.x & 0xFFFFu);
        dm[r] = h2f(hd.x >> 16);
        // 6-bit scales and mins of sub-blocks 0..3 (p < 2) or 4..7, four per word
        uint32_t scw, mw;
        if (p < 2) {
            scw = hd.y & 0x3F3F3F3Fu;
            mw = hd.z & 0x3F3F3F3Fu;
        } else {
            scw = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
            mw = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        }
        const int sh = 16 * (p & 1);
        sc0[r] = float((scw >> sh) & 0xFFu);
        sc1[r] = float((scw >> (sh + 8)) & 0xFFu);
        m0[r] = float((mw >> sh) & 0xFFu);
        m1[r] = float((mw >> (sh + 8)) & 0xFFu);
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 64 * p + 16 * h;
        const int4 xa = ldx16(P.xq + o), xb = ldx16(P.xq + o + 32);
        const int4 ya = ldx16(P.xq2 + o), yb = ldx16(P.xq2 + o + 32);
        const long long g = ((tk.tb[t] + (long long)sb * 256) >> 5) + 2 * p;
        const float2 dd = __ldg(reinterpret_cast<const float2*>(P.xd + g));
        const float2 ss = __ldg(reinterpret_cast<const float2*>(P.xs + g));
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s0 = dp4(lo[r][0], xa.x, 0); s0 = dp4(lo[r][1], xa.y, s0); s0 = dp4(lo[r][2], xa.z, s0); s0 = dp4(lo[r][3], xa.w, s0);
            int s1 = dp4(hi[r][0], xb.x, 0); s1 = dp4(hi[r][1], xb.y, s1); s1 = dp4(hi[r][2], xb.z, s1); s1 = dp4(hi[r][3], xb.w, s1);
            int u0 = dp4(lo[r][0], ya.x, 0); u0 = dp4(lo[r][1], ya.y, u0); u0 = dp4(lo[r][2], ya.z, u0); u0 = dp4(lo[r][3], ya.w, u0);
            int u1 = dp4(hi[r][0], yb.x, 0); u1 = dp4(hi[r][1], yb.y, u1); u1 = dp4(hi[r][2], yb.z, u1); u1 = dp4(hi[r][3], yb.w, u1);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + 2 * p;
                atomicAdd(P.s + base, s0); atomicAdd(P.s + base + 1, s1);
                atomicAdd(P.s2 + base, u0); atomicAdd(P.s2 + base + 1, u1);
            } else {
                float a = d[r] * (dd.x * sc0[r] * (float(s0) + float(u0) * kInv254)
                                  + dd.y * sc1[r] * (float(s1) + float(u1) * kInv254));
                if (h == 0) a -= dm[r] * (m0[r] * ss.x + m1[r] * ss.y);    // the min term once per sub-block
                acc[r][t] += a;
            }
        }
    }
}

// ---- Q6_K: 210 B = ql[128], qh[64], int8 scales[16], d (f16) (quant.py:140-159).  Half n holds 128
// values; group g (0..3) of 32: low 4 bits from ql[64n + 32(g&1) + l] (nibble g>>1), top 2 bits from
// qh[32n + l] bits 2g.  Lane q (n = q/4, j = q%4) takes ql bytes 64n+16j..+15: groups A = j/2 (low
// nibble) and A+2 (high nibble), l = 16(j%2)..+15; one int8 scale per 16 values.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_q6k(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int n = q >> 2, j = q & 3, A = j >> 1, B = A + 2, l0 = 16 * (j & 1);
    uint32_t wa[RW][4], wb[RW][4];
    float d[RW], sa[RW], sbs[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 210;
        const uint4 ql = ldw16_a2(b + 64 * n + 16 * j);
        const uint4 qh = ldw16_a2(b + 128 + 32 * n + l0);
        sa[r] = float(int8_t(ldw1(b + 192 + 8 * n + 2 * A + (j & 1))));
        sbs[r] = float(int8_t(ldw1(b + 192 + 8 * n + 2 * B + (j & 1))));
        d[r] = h2f(ldw2(b + 208));
        const uint32_t L[4] = {ql.x, ql.y, ql.z, ql.w}, H[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            wa[r][i] = __vsub4((L[i] & 0x0F0F0F0Fu) | (((H[i] >> (2 * A)) & 0x03030303u) << 4), 0x20202020u);
            wb[r][i] = __vsub4(((L[i] >> 4) & 0x0F0F0F0Fu) | (((H[i] >> (2 * B)) & 0x03030303u) << 4), 0x20202020u);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 128 * n + l0;
        const int4 xa = ldx16(P.xq + o + 32 * A), xb = ldx16(P.xq + o + 32 * B);
        const int4 ya = ldx16(P.xq2 + o + 32 * A), yb = ldx16(P.xq2 + o + 32 * B);
        const long long g = ((tk.tb[t] + (long long)sb * 256) >> 5) + 4 * n;
        const float da = __ldg(P.xd + g + A), db = __ldg(P.xd + g + B);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s0 = dp4(wa[r][0], xa.x, 0); s0 = dp4(wa[r][1], xa.y, s0); s0 = dp4(wa[r][2], xa.z, s0); s0 = dp4(wa[r][3], xa.w, s0);
            int s1 = dp4(wb[r][0], xb.x, 0); s1 = dp4(wb[r][1], xb.y, s1); s1 = dp4(wb[r][2], xb.z, s1); s1 = dp4(wb[r][3], xb.w, s1);
            int u0 = dp4(wa[r][0], ya.x, 0); u0 = dp4(wa[r][1], ya.y, u0); u0 = dp4(wa[r][2], ya.z, u0); u0 = dp4(wa[r][3], ya.w, u0);
            int u1 = dp4(wb[r][0], yb.x, 0); u1 = dp4(wb[r][1], yb.y, u1); u1 = dp4(wb[r][2], yb.z, u1); u1 = dp4(wb[r][3], yb.w, u1);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 16) + sb * 16 + 8 * n + (j & 1);
                atomicAdd(P.s + base + 2 * A, s0); atomicAdd(P.s + base + 2 * B, s1);
                atomicAdd(P.s2 + base + 2 * A, u0); atomicAdd(P.s2 + base + 2 * B, u1);
            } else {
                acc[r][t] += d[r] * (sa[r] * da * (float(s0) + float(u0) * kInv254)
                                     + sbs[r] * db * (float(s1) + float(u1) * kInv254));
            }
        }
    }
}

// ---- Q4_0: 18 B = d (f16), 16 B nibbles: low nibble = value i, high = value 16+i (quant.py:60-64).
// Lane q takes block 8*sb + q of the row; the code is the unsigned nibble, the -8 goes with xs.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_q4_0(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                          const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int blk = sb * 8 + q;
    if (blk >= P.n_in / 32) return;
    uint32_t lo[RW][4], hi[RW][4];
    float d[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)blk * 18;
        d[r] = h2f(ldw2(b));
        const uint4 v = ldw16_a2(b + 2);
        lo[r][0] = v.x & 0x0F0F0F0Fu; hi[r][0] = (v.x >> 4) & 0x0F0F0F0Fu;
        lo[r][1] = v.y & 0x0F0F0F0Fu; hi[r][1] = (v.y >> 4) & 0x0F0F0F0Fu;
        lo[r][2] = v.z & 0x0F0F0F0Fu; hi[r][2] = (v.z >> 4) & 0x0F0F0F0Fu;
        lo[r][3] = v.w & 0x0F0F0F0Fu; hi[r][3] = (v.w >> 4) & 0x0F0F0F0Fu;
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)blk * 32;
        const int4 xa = ldx16(P.xq + o), xb = ldx16(P.xq + o + 16);
        const int4 ya = ldx16(P.xq2 + o), yb = ldx16(P.xq2 + o + 16);
        const long long g = (tk.tb[t] >> 5) + blk;
        const float dd = __ldg(P.xd + g), ss = __ldg(P.xs + g);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(lo[r][0], xa.x, 0); s = dp4(lo[r][1], xa.y, s); s = dp4(lo[r][2], xa.z, s); s = dp4(lo[r][3], xa.w, s);
            s = dp4(hi[r][0], xb.x, s); s = dp4(hi[r][1], xb.y, s); s = dp4(hi[r][2], xb.z, s); s = dp4(hi[r][3], xb.w, s);
            int u = dp4(lo[r][0], ya.x, 0); u = dp4(lo[r][1], ya.y, u); u = dp4(lo[r][2], ya.z, u); u = dp4(lo[r][3], ya.w, u);
            u = dp4(hi[r][0], yb.x, u); u = dp4(hi[r][1], yb.y, u); u = dp4(hi[r][2], yb.z, u); u = dp4(hi[r][3], yb.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + blk;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += d[r] * (dd * (float(s) + float(u) * kInv254) - 8.0f * ss);
            }
        }
    }
}

// ---- Q4_1 (20 B: d, m, 16 B nibbles), Q5_0 (22 B: d, qh u32, nibbles), Q5_1 (24 B: d, m, qh, nibbles),
// IQ4_NL (18 B: d, 16 B codebook indices); byte j holds values j (low nibble) and 16 + j, bit j of qh is
// bit 4 of value j (quant.py:67-95, 264-270).  Lane q takes block 8*sb + q.  Unsigned codes for the
// Q4_1 / Q5_x formats: y = d xd (S + S2/254) - off xs with off = -m (Q4_1, Q5_1) or 16 d (Q5_0).
template <int FMT>
__device__ __forceinline__ void b32_codes(const uint8_t* b, uint32_t (&lo)[4], uint32_t (&hi)[4], float& d, float& off) {
    d = h2f(ldw2(b));
    constexpr int qo = FMT == F_Q4_1 ? 4 : FMT == F_Q5_0 ? 6 : FMT == F_Q5_1 ? 8 : 2;
    const uint4 v = ldw16_a2(b + qo);
    const uint32_t V[4] = {v.x, v.y, v.z, v.w};
    uint32_t qh = 0u;
    if constexpr (FMT == F_Q5_0) qh = ldw2(b + 2) | (ldw2(b + 4) << 16);
    if constexpr (FMT == F_Q5_1) qh = ldw2(b + 4) | (ldw2(b + 6) << 16);
    off = FMT == F_Q5_0 ? 16.0f * d : (FMT == F_Q4_1 || FMT == F_Q5_1) ? -h2f(ldw2(b + 2)) : 0.f;
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
}

template <int FMT, int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_b32(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int blk = sb * 8 + q;
    if (blk >= P.n_in / 32) return;
    uint32_t lo[RW][4], hi[RW][4];
    float d[RW], off[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) b32_codes<FMT>(rows[r] + (long long)blk * block_bytes(FMT), lo[r], hi[r], d[r], off[r]);
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)blk * 32;
        const int4 xa = ldx16(P.xq + o), xb = ldx16(P.xq + o + 16);
        const int4 ya = ldx16(P.xq2 + o), yb = ldx16(P.xq2 + o + 16);
        const long long g = (tk.tb[t] >> 5) + blk;
        const float dd = __ldg(P.xd + g), ss = __ldg(P.xs + g);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(lo[r][0], xa.x, 0); s = dp4(lo[r][1], xa.y, s); s = dp4(lo[r][2], xa.z, s); s = dp4(lo[r][3], xa.w, s);
            s = dp4(hi[r][0], xb.x, s); s = dp4(hi[r][1], xb.y, s); s = dp4(hi[r][2], xb.z, s); s = dp4(hi[r][3], xb.w, s);
            int u = dp4(lo[r][0], ya.x, 0); u = dp4(lo[r][1], ya.y, u); u = dp4(lo[r][2], ya.z, u); u = dp4(lo[r][3], ya.w, u);
            u = dp4(hi[r][0], yb.x, u); u = dp4(hi[r][1], yb.y, u); u = dp4(hi[r][2], yb.z, u); u = dp4(hi[r][3], yb.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + blk;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += d[r] * dd * (float(s) + float(u) * kInv254) - off[r] * ss;
            }
        }
    }
}

// ---- Q1_0 (128 values: d, 16 B of bits, value j = bit j % 8 of byte j / 8: d (2 b - 1)), Q2_0 (64 values:
// d, 16 B) and PQ2_0 (128 values: d, 32 B) with value j at bits 2 (j % 4) of byte j / 4: d (q - 1)
// (quant.py:406-428).  Lane q takes the 32-value unit 8*sb + q.  Q1_0 codes are the bits (weight scale
// 2 d, offset d xs); Q2_0 codes q (offset d xs) meet the activation bytes transposed 4 x 4.
template <int FMT>
__device__ __forceinline__ const uint8_t* bits_unit(const uint8_t* row, int u, int& sub) {
    constexpr int upb = block_values(FMT) / 32;
    sub = u % upb;
    return row + (long long)(u / upb) * block_bytes(FMT);
}
template <int T, int RW, bool SUMS, int FMT>
__device__ __forceinline__ void lane_bits(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                          const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int u = sb * 8 + q;
    if (u >= P.n_in / 32) return;
    uint32_t w[RW][8];
    float d[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        int sub;
        const uint8_t* b = bits_unit<FMT>(rows[r], u, sub);
        d[r] = h2f(ldw2(b));
        if constexpr (FMT == F_Q1_0) {
            const uint32_t bits = ldw2(b + 2 + 4 * sub) | (ldw2(b + 4 + 4 * sub) << 16);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                w[r][2 * k] = spread4(bits >> (8 * k));
                w[r][2 * k + 1] = spread4(bits >> (8 * k + 4));
            }
        } else {
            const uint2 c = ldw8_a2(b + 2 + 8 * sub);
#pragma unroll
            for (int s = 0; s < 4; ++s) {
                w[r][s] = (c.x >> (2 * s)) & 0x03030303u;
                w[r][4 + s] = (c.y >> (2 * s)) & 0x03030303u;
            }
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)u * 32;
        int4 xa = ldx16(P.xq + o), xb = ldx16(P.xq + o + 16);
        int4 ya = ldx16(P.xq2 + o), yb = ldx16(P.xq2 + o + 16);
        if constexpr (FMT != F_Q1_0) {
            xa = byte_transpose(xa); xb = byte_transpose(xb);
            ya = byte_transpose(ya); yb = byte_transpose(yb);
        }
        const long long g = (tk.tb[t] >> 5) + u;
        const float dd = __ldg(P.xd + g), ss = __ldg(P.xs + g);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], xa.x, 0); s = dp4(w[r][1], xa.y, s); s = dp4(w[r][2], xa.z, s); s = dp4(w[r][3], xa.w, s);
            s = dp4(w[r][4], xb.x, s); s = dp4(w[r][5], xb.y, s); s = dp4(w[r][6], xb.z, s); s = dp4(w[r][7], xb.w, s);
            int v = dp4(w[r][0], ya.x, 0); v = dp4(w[r][1], ya.y, v); v = dp4(w[r][2], ya.z, v); v = dp4(w[r][3], ya.w, v);
            v = dp4(w[r][4], yb.x, v); v = dp4(w[r][5], yb.y, v); v = dp4(w[r][6], yb.z, v); v = dp4(w[r][7], yb.w, v);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + u;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, v);
            } else {
                const float wsc = FMT == F_Q1_0 ? 2.0f * d[r] : d[r];
                acc[r][t] += wsc * dd * (float(s) + float(v) * kInv254) - d[r] * ss;
            }
        }
    }
}

// ---- Q3_K: 110 B = hmask[32], qs[64], scales[12], d (f16) (quant.py:295-306).  Lane q takes values
// 32q..32q+31 of the superblock: half n = q/4, 2-bit field s = q%4 of qs[32n + l], high bit q of hmask[l];
// scale group 2q (values 0..15) and 2q + 1 (16..31): 6-bit scale (nibble of scales[i % 8], 2 bits of
// scales[8 + i % 4]) - 32.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_q3k(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int n = q >> 2, s2 = 2 * (q & 3);
    uint32_t w[RW][8];
    float sc0[RW], sc1[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 110;
        const uint4 q0 = ldw16_a2(b + 32 + 32 * n), q1 = ldw16_a2(b + 48 + 32 * n);
        const uint4 h0 = ldw16_a2(b), h1 = ldw16_a2(b + 16);
        const uint32_t Q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        const uint32_t H[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) w[r][i] = q3k_word((Q[i] >> s2) & 0x03030303u, (H[i] >> q) & 0x01010101u);
        const float d = h2f(ldw2(b + 108));
        const int i0 = 2 * q, i1 = 2 * q + 1;
        const int l0 = int(ldw1(b + 96 + i0 % 8) >> (4 * (i0 / 8))) & 15, g0 = int(ldw1(b + 104 + i0 % 4) >> (2 * (i0 / 4))) & 3;
        const int l1 = int(ldw1(b + 96 + i1 % 8) >> (4 * (i1 / 8))) & 15, g1 = int(ldw1(b + 104 + i1 % 4) >> (2 * (i1 / 4))) & 3;
        sc0[r] = d * float((l0 | (g0 << 4)) - 32);
        sc1[r] = d * float((l1 | (g1 << 4)) - 32);
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int sa = dp4(w[r][0], x0.x, 0); sa = dp4(w[r][1], x0.y, sa); sa = dp4(w[r][2], x0.z, sa); sa = dp4(w[r][3], x0.w, sa);
            int sb2 = dp4(w[r][4], x1.x, 0); sb2 = dp4(w[r][5], x1.y, sb2); sb2 = dp4(w[r][6], x1.z, sb2); sb2 = dp4(w[r][7], x1.w, sb2);
            int ua = dp4(w[r][0], y0.x, 0); ua = dp4(w[r][1], y0.y, ua); ua = dp4(w[r][2], y0.z, ua); ua = dp4(w[r][3], y0.w, ua);
            int ub = dp4(w[r][4], y1.x, 0); ub = dp4(w[r][5], y1.y, ub); ub = dp4(w[r][6], y1.z, ub); ub = dp4(w[r][7], y1.w, ub);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 16) + sb * 16 + 2 * q;
                atomicAdd(P.s + base, sa); atomicAdd(P.s + base + 1, sb2);
                atomicAdd(P.s2 + base, ua); atomicAdd(P.s2 + base + 1, ub);
            } else {
                acc[r][t] += dd * (sc0[r] * (float(sa) + float(ua) * kInv254) + sc1[r] * (float(sb2) + float(ub) * kInv254));
            }
        }
    }
}

// ---- IQ2_XS (74 B = d, u16 qs[32], scales[8]) and IQ2_S (82 B = d, qs[32], signs[32], qh[8], scales[8])
// (quant.py:248-260, 310-318).  Entry k (8 values): IQ2_XS index bits 0..8 of qs[k] with a 7-bit sign
// index in bits 9..15 (parity gives the 8th sign); IQ2_S index qs[k] | bits 2 (k % 4).. of qh[k / 4] << 8
// with sign byte signs[k].  The 16-value scale group i has weight scale d (0.125 + 0.25 s), s = nibble
// i % 2 of scales[i / 2].  Codebooks compact (2 bits per magnitude) in global memory, read through L1.
__device__ const uint16_t kIq2xsCodes[512] = {
#include "iq2xs_grid.inc"
};
__device__ const uint16_t kIq2sCodes[1024] = {
#include "iq2s_grid.inc"
};

// the signed bytes of sub-block q (entries 4q..4q+3) of an IQ2_XS / IQ2_S block at b (global or shared
// through the loader L), and the two scale nibbles
template <int FMT>
__device__ __forceinline__ void iq2x_words(uint32_t q0, uint32_t q1, uint32_t sg, uint32_t qh, uint32_t (&w)[8]) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        uint32_t idx, s8;
        if constexpr (FMT == F_IQ2_XS) {
            const uint32_t q16 = ((e < 2 ? q0 : q1) >> (16 * (e & 1))) & 0xFFFFu;
            idx = q16 & 511u;
            const uint32_t s7 = q16 >> 9;
            s8 = s7 | (uint32_t(__popc(s7) & 1) << 7);
        } else {
            idx = ((q0 >> (8 * e)) & 0xFFu) | (((qh >> (2 * e)) & 3u) << 8);
            s8 = (sg >> (8 * e)) & 0xFFu;
        }
        const uint32_t code = FMT == F_IQ2_XS ? uint32_t(__ldg(kIq2xsCodes + idx)) : uint32_t(__ldg(kIq2sCodes + idx));
        const uint32_t mlo = sign4_mask(s8), mhi = sign4_mask(s8 >> 4);
        w[2 * e] = __vsub4(iq2_mag4(code & 0xFFu) ^ mlo, mlo);
        w[2 * e + 1] = __vsub4(iq2_mag4(code >> 8) ^ mhi, mhi);
    }
}

template <int T, int RW, bool SUMS, int FMT>
__device__ __forceinline__ void lane_iq2x(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                          const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    uint32_t w[RW][8];
    float sc0[RW], sc1[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * block_bytes(FMT);
        uint32_t q0, q1 = 0u, sg = 0u, qh = 0u, scb;
        if constexpr (FMT == F_IQ2_XS) {
            const uint2 c = ldw8_a2(b + 2 + 8 * q);
            q0 = c.x;
            q1 = c.y;
            scb = ldw1(b + 66 + q);
        } else {
            q0 = ldw2(b + 2 + 4 * q) | (ldw2(b + 4 + 4 * q) << 16);
            sg = ldw2(b + 34 + 4 * q) | (ldw2(b + 36 + 4 * q) << 16);
            qh = ldw1(b + 66 + q);
            scb = ldw1(b + 74 + q);
        }
        iq2x_words<FMT>(q0, q1, sg, qh, w[r]);
        const float d = h2f(ldw2(b));
        sc0[r] = d * (0.125f + 0.25f * float(scb & 15u));
        sc1[r] = d * (0.125f + 0.25f * float(scb >> 4));
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int sa = dp4(w[r][0], x0.x, 0); sa = dp4(w[r][1], x0.y, sa); sa = dp4(w[r][2], x0.z, sa); sa = dp4(w[r][3], x0.w, sa);
            int sb2 = dp4(w[r][4], x1.x, 0); sb2 = dp4(w[r][5], x1.y, sb2); sb2 = dp4(w[r][6], x1.z, sb2); sb2 = dp4(w[r][7], x1.w, sb2);
            int ua = dp4(w[r][0], y0.x, 0); ua = dp4(w[r][1], y0.y, ua); ua = dp4(w[r][2], y0.z, ua); ua = dp4(w[r][3], y0.w, ua);
            int ub = dp4(w[r][4], y1.x, 0); ub = dp4(w[r][5], y1.y, ub); ub = dp4(w[r][6], y1.z, ub); ub = dp4(w[r][7], y1.w, ub);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 16) + sb * 16 + 2 * q;
                atomicAdd(P.s + base, sa); atomicAdd(P.s + base + 1, sb2);
                atomicAdd(P.s2 + base, ua); atomicAdd(P.s2 + base + 1, ub);
            } else {
                acc[r][t] += dd * (sc0[r] * (float(sa) + float(ua) * kInv254) + sc1[r] * (float(sb2) + float(ub) * kInv254));
            }
        }
    }
}

// ---- Q2_K: 84 B = scales[16] (low nibble: scale, high: min), qs[64], d, dmin (quant.py:284-292).  Lane q
// takes values 32q..32q+31: 2-bit field 2 (q % 4) of qs[32 (q / 4) + l]; 16-value groups 2q, 2q + 1 with
// weight scale d sc and minimum dmin m.  The minimum multiplies the quantised input's own 16-value sum,
// xd (sum xq + sum xq2 / 254): xs covers 32 values, the minimum only 16.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_q2k(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int n = q >> 2, s2 = 2 * (q & 3);
    uint32_t w[RW][8];
    float dl0[RW], dl1[RW], ml0[RW], ml1[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 84;
        const uint4 q0 = ldw16_a2(b + 16 + 32 * n), q1 = ldw16_a2(b + 32 + 32 * n);
        const uint32_t Q[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) w[r][i] = (Q[i] >> s2) & 0x03030303u;
        const float d = h2f(ldw2(b + 80)), dm = h2f(ldw2(b + 82));
        const uint32_t sc0 = ldw1(b + 2 * q), sc1 = ldw1(b + 2 * q + 1);
        dl0[r] = d * float(sc0 & 15u); ml0[r] = dm * float(sc0 >> 4);
        dl1[r] = d * float(sc1 & 15u); ml1[r] = dm * float(sc1 >> 4);
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
        constexpr uint32_t one = 0x01010101u;
        const int qa = dp4(one, x0.w, dp4(one, x0.z, dp4(one, x0.y, dp4(one, x0.x, 0))));
        const int qb = dp4(one, x1.w, dp4(one, x1.z, dp4(one, x1.y, dp4(one, x1.x, 0))));
        const int ra = dp4(one, y0.w, dp4(one, y0.z, dp4(one, y0.y, dp4(one, y0.x, 0))));
        const int rb = dp4(one, y1.w, dp4(one, y1.z, dp4(one, y1.y, dp4(one, y1.x, 0))));
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int sa = dp4(w[r][0], x0.x, 0); sa = dp4(w[r][1], x0.y, sa); sa = dp4(w[r][2], x0.z, sa); sa = dp4(w[r][3], x0.w, sa);
            int sb2 = dp4(w[r][4], x1.x, 0); sb2 = dp4(w[r][5], x1.y, sb2); sb2 = dp4(w[r][6], x1.z, sb2); sb2 = dp4(w[r][7], x1.w, sb2);
            int ua = dp4(w[r][0], y0.x, 0); ua = dp4(w[r][1], y0.y, ua); ua = dp4(w[r][2], y0.z, ua); ua = dp4(w[r][3], y0.w, ua);
            int ub = dp4(w[r][4], y1.x, 0); ub = dp4(w[r][5], y1.y, ub); ub = dp4(w[r][6], y1.z, ub); ub = dp4(w[r][7], y1.w, ub);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 16) + sb * 16 + 2 * q;
                atomicAdd(P.s + base, sa); atomicAdd(P.s + base + 1, sb2);
                atomicAdd(P.s2 + base, ua); atomicAdd(P.s2 + base + 1, ub);
            } else {
                acc[r][t] += dd * (dl0[r] * (float(sa) + float(ua) * kInv254) + dl1[r] * (float(sb2) + float(ub) * kInv254)
                                   - ml0[r] * (float(qa) + float(ra) * kInv254) - ml1[r] * (float(qb) + float(rb) * kInv254));
            }
        }
    }
}

// ---- TQ1_0: 54 B = qs[48], qh[4], d (quant.py:405-458).  Five trits per byte as a fixed-point fraction:
// trit n of byte v = ((v 3^n) mod 256) 3 >> 8.  Values 0..159: byte j % 32, n = j / 32; 160..239: byte
// 32 + (j - 160) % 16, n = (j - 160) / 16; 240..255: byte 48 + (j - 240) % 4, n = (j - 240) / 4.  Lane q
// takes values 32q..32q+31; every four consecutive values share one power, so the trits of a word come
// out together (bytes multiplied in 16-bit lanes).  The code is the trit, value d (trit - 1): offset d xs.
__device__ __forceinline__ uint32_t trits4(uint32_t w, uint32_t pw) {
    const uint32_t lo = ((w & 0x00FF00FFu) * pw) & 0x00FF00FFu, hi = (((w >> 8) & 0x00FF00FFu) * pw) & 0x00FF00FFu;
    return (((lo * 3u) >> 8) & 0x00030003u) | ((((hi * 3u) >> 8) & 0x00030003u) << 8);
}
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_tq1(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    uint32_t w[RW][8];
    float d[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 54;
        d[r] = h2f(ldw2(b + 52));
        if (q < 5) {
            const uint32_t pw = q == 0 ? 1u : q == 1 ? 3u : q == 2 ? 9u : q == 3 ? 27u : 81u;
            const uint4 a0 = ldw16_a2(b), a1 = ldw16_a2(b + 16);
            const uint32_t V[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) w[r][i] = trits4(V[i], pw);
        } else {
            const uint4 a = ldw16_a2(b + 32);
            const uint32_t V[4] = {a.x, a.y, a.z, a.w};
            const uint32_t p0 = q == 5 ? 1u : q == 6 ? 9u : 81u, p1 = q == 5 ? 3u : 27u;
#pragma unroll
            for (int i = 0; i < 4; ++i) w[r][i] = trits4(V[i], p0);
            if (q < 7) {
#pragma unroll
                for (int i = 0; i < 4; ++i) w[r][4 + i] = trits4(V[i], p1);
            } else {
                const uint32_t h = ldw2(b + 48) | (ldw2(b + 50) << 16);
                w[r][4] = trits4(h, 1u); w[r][5] = trits4(h, 3u); w[r][6] = trits4(h, 9u); w[r][7] = trits4(h, 27u);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const long long g = ((tk.tb[t] + (long long)sb * 256) >> 5) + q;
        const float dd = __ldg(P.xd + g), ss = __ldg(P.xs + g);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], x0.x, 0); s = dp4(w[r][1], x0.y, s); s = dp4(w[r][2], x0.z, s); s = dp4(w[r][3], x0.w, s);
            s = dp4(w[r][4], x1.x, s); s = dp4(w[r][5], x1.y, s); s = dp4(w[r][6], x1.z, s); s = dp4(w[r][7], x1.w, s);
            int u = dp4(w[r][0], y0.x, 0); u = dp4(w[r][1], y0.y, u); u = dp4(w[r][2], y0.z, u); u = dp4(w[r][3], y0.w, u);
            u = dp4(w[r][4], y1.x, u); u = dp4(w[r][5], y1.y, u); u = dp4(w[r][6], y1.z, u); u = dp4(w[r][7], y1.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + q;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += d[r] * (dd * (float(s) + float(u) * kInv254) - ss);
            }
        }
    }
}

// ---- IQ1_S (50 B = d, qs[32], qh u16[8]; quant.py:350-360) and IQ1_M (56 B = qs[32], qh[16], scales
// u16[4]; quant.py:363-375).  Lane q takes sub-block q: codebook entries 4q..4q+3, eight values each in
// {-1, 0, +1} (kIq1sCodes, two bits a value) plus a delta of +-1/8 per sub-block (IQ1_S) or per entry
// (IQ1_M).  Value = dl (g + delta) with dl = d (2 s + 1): the code 8 g +- 1 is an exact int8 and the weight
// scale dl / 8, so the sums need nothing but xq / xq2.  IQ1_M's 3-bit scales cover 16 values (two groups
// per lane) and its d sits in the top nibbles of the four scale words.
__device__ const uint16_t kIq1sCodes[2048] = {
#include "iq1s_grid.inc"
};
// eight codes 8 g + (neg ? -1 : +1) of one codebook entry as two words of int8 bytes
__device__ __forceinline__ void iq1_words(uint32_t idx, uint32_t neg, uint32_t& lo, uint32_t& hi) {
    const uint32_t c = __ldg(kIq1sCodes + idx);
    const uint32_t delta = neg ? 0xFFFFFFFFu : 0x01010101u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t c4 = (c >> (8 * h)) & 0xFFu;
        const uint32_t f = (c4 | (c4 << 6) | (c4 << 12) | (c4 << 18)) & 0x03030303u;   // 2-bit field per byte
        const uint32_t g8 = __vsub4((f & 0x01010101u) << 3, (f & 0x02020202u) << 3);   // 8 g: 0, 8 or -8
        (h ? hi : lo) = __vadd4(g8, delta);
    }
}
__device__ __forceinline__ float iq1m_d(const uint8_t* b) {
    const uint32_t s01 = ldw2(b + 48) | (ldw2(b + 50) << 16), s23 = ldw2(b + 52) | (ldw2(b + 54) << 16);
    const uint32_t d16 = ((s01 >> 12) & 0xFu) | ((s01 >> 24) & 0xF0u) | ((s23 >> 4) & 0xF00u) | ((s23 >> 16) & 0xF000u);
    return h2f(d16);
}
template <int T, int RW, bool SUMS, int FMT>
__device__ __forceinline__ void lane_iq1(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    uint32_t w[RW][8];
    float wsc[RW][2];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * block_bytes(FMT);
        if constexpr (FMT == F_IQ1_S) {
            const uint32_t qh = ldw2(b + 34 + 2 * q);
            const uint32_t qs = ldw2(b + 2 + 4 * q) | (ldw2(b + 4 + 4 * q) << 16);
#pragma unroll
            for (int l = 0; l < 4; ++l)
                iq1_words(((qs >> (8 * l)) & 0xFFu) | (((qh >> (3 * l)) & 7u) << 8), qh >> 15, w[r][2 * l], w[r][2 * l + 1]);
            wsc[r][0] = wsc[r][1] = h2f(ldw2(b)) * (float(2 * ((qh >> 12) & 7u) + 1) * 0.125f);
        } else {
            const uint32_t qs = ldw2(b + 4 * q) | (ldw2(b + 2 + 4 * q) << 16);
            const uint32_t nb = ldw2(b + 32 + 2 * q);              // nibbles of entries 4q..4q+3
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const uint32_t nib = (nb >> (4 * l)) & 15u;
                iq1_words(((qs >> (8 * l)) & 0xFFu) | ((nib & 7u) << 8), nib >> 3, w[r][2 * l], w[r][2 * l + 1]);
            }
            const float d = iq1m_d(b);
            const uint32_t sw = ldw2(b + 48 + 2 * (q >> 1));       // groups 2q, 2q + 1: fields (2q) % 4, (2q+1) % 4
#pragma unroll
            for (int k = 0; k < 2; ++k)
                wsc[r][k] = d * (float(2 * ((sw >> (3 * ((2 * q + k) & 3))) & 7u) + 1) * 0.125f);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            const int s0 = dp4(w[r][3], x0.w, dp4(w[r][2], x0.z, dp4(w[r][1], x0.y, dp4(w[r][0], x0.x, 0))));
            const int s1 = dp4(w[r][7], x1.w, dp4(w[r][6], x1.z, dp4(w[r][5], x1.y, dp4(w[r][4], x1.x, 0))));
            const int u0 = dp4(w[r][3], y0.w, dp4(w[r][2], y0.z, dp4(w[r][1], y0.y, dp4(w[r][0], y0.x, 0))));
            const int u1 = dp4(w[r][7], y1.w, dp4(w[r][6], y1.z, dp4(w[r][5], y1.y, dp4(w[r][4], y1.x, 0))));
            if constexpr (SUMS) {
                if constexpr (FMT == F_IQ1_S) {
                    const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + q;
                    atomicAdd(P.s + base, s0 + s1);
                    atomicAdd(P.s2 + base, u0 + u1);
                } else {
                    const long long base = (long long)row0 * (P.n_in / 16) + sb * 16 + 2 * q;
                    atomicAdd(P.s + base, s0);
                    atomicAdd(P.s2 + base, u0);
                    atomicAdd(P.s + base + 1, s1);
                    atomicAdd(P.s2 + base + 1, u1);
                }
            } else {
                acc[r][t] += dd * (wsc[r][0] * (float(s0) + float(u0) * kInv254) +
                                   wsc[r][1] * (float(s1) + float(u1) * kInv254));
            }
        }
    }
}

// ---- PTQ1_0 (28 B = qs[24], qh[2], d; quant.py:431-469, trit_plan(24, 2)): values 0..79 are trit j / 16 of
// byte j % 16, 80..119 trit (j - 80) / 8 of byte 16 + (j - 80) % 8, 120..127 trit (j - 120) / 2 of qh byte
// (j - 120) % 2.  Lane q takes the 32-value unit 8 sb + q (unit u % 4 of block u / 4); the code is the trit,
// value d (trit - 1): offset d xs.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_ptq1(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                          const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int u = sb * 8 + q;
    if (u >= P.n_in / 32) return;
    const int sub = u & 3;
    uint32_t w[RW][8];
    float d[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)(u >> 2) * 28;
        d[r] = h2f(ldw2(b + 26));
        const uint4 a = ldw16_a2(b);                           // bytes 0..15
        const uint2 c = ldw8_a2(b + 16);                       // bytes 16..23
        const uint32_t A[4] = {a.x, a.y, a.z, a.w};
        if (sub < 2) {                                         // values 32 sub ..: powers 3^(2 sub), 3^(2 sub + 1)
            const uint32_t p0 = sub == 0 ? 1u : 9u, p1 = sub == 0 ? 3u : 27u;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                w[r][i] = trits4(A[i], p0);
                w[r][4 + i] = trits4(A[i], p1);
            }
        } else if (sub == 2) {                                 // 64..79: 3^4 of bytes 0..15; 80..95: 3^0, 3^1 of 16..23
#pragma unroll
            for (int i = 0; i < 4; ++i) w[r][i] = trits4(A[i], 81u);
            w[r][4] = trits4(c.x, 1u); w[r][5] = trits4(c.y, 1u);
            w[r][6] = trits4(c.x, 3u); w[r][7] = trits4(c.y, 3u);
        } else {                                               // 96..119: 3^2..3^4 of 16..23; 120..127: qh
            w[r][0] = trits4(c.x, 9u); w[r][1] = trits4(c.y, 9u);
            w[r][2] = trits4(c.x, 27u); w[r][3] = trits4(c.y, 27u);
            w[r][4] = trits4(c.x, 81u); w[r][5] = trits4(c.y, 81u);
            const uint32_t h = ldw2(b + 24);
            const uint32_t hh = h | (h << 16);                 // bytes qh0, qh1, qh0, qh1
            w[r][6] = (trits4(hh, 1u) & 0x0000FFFFu) | (trits4(hh, 3u) & 0xFFFF0000u);
            w[r][7] = (trits4(hh, 9u) & 0x0000FFFFu) | (trits4(hh, 27u) & 0xFFFF0000u);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)u * 32;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const long long g = (tk.tb[t] >> 5) + u;
        const float dd = __ldg(P.xd + g), ss = __ldg(P.xs + g);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], x0.x, 0); s = dp4(w[r][1], x0.y, s); s = dp4(w[r][2], x0.z, s); s = dp4(w[r][3], x0.w, s);
            s = dp4(w[r][4], x1.x, s); s = dp4(w[r][5], x1.y, s); s = dp4(w[r][6], x1.z, s); s = dp4(w[r][7], x1.w, s);
            int v = dp4(w[r][0], y0.x, 0); v = dp4(w[r][1], y0.y, v); v = dp4(w[r][2], y0.z, v); v = dp4(w[r][3], y0.w, v);
            v = dp4(w[r][4], y1.x, v); v = dp4(w[r][5], y1.y, v); v = dp4(w[r][6], y1.z, v); v = dp4(w[r][7], y1.w, v);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + u;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, v);
            } else {
                acc[r][t] += d[r] * (dd * (float(s) + float(v) * kInv254) - ss);
            }
        }
    }
}

// ---- Q8_0: 34 B = d (f16), int8[32] (quant.py:46-50).  Lane q takes block 8*sb + q.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_q8_0(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                          const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int blk = sb * 8 + q;
    if (blk >= P.n_in / 32) return;
    uint32_t w[RW][8];
    float d[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)blk * 34;
        d[r] = h2f(ldw2(b));
        const uint4 v0 = ldw16_a2(b + 2), v1 = ldw16_a2(b + 18);
        w[r][0] = v0.x; w[r][1] = v0.y; w[r][2] = v0.z; w[r][3] = v0.w;
        w[r][4] = v1.x; w[r][5] = v1.y; w[r][6] = v1.z; w[r][7] = v1.w;
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)blk * 32;
        const int4 xa = ldx16(P.xq + o), xb = ldx16(P.xq + o + 16);
        const int4 ya = ldx16(P.xq2 + o), yb = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + (tk.tb[t] >> 5) + blk);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], xa.x, 0); s = dp4(w[r][1], xa.y, s); s = dp4(w[r][2], xa.z, s); s = dp4(w[r][3], xa.w, s);
            s = dp4(w[r][4], xb.x, s); s = dp4(w[r][5], xb.y, s); s = dp4(w[r][6], xb.z, s); s = dp4(w[r][7], xb.w, s);
            int u = dp4(w[r][0], ya.x, 0); u = dp4(w[r][1], ya.y, u); u = dp4(w[r][2], ya.z, u); u = dp4(w[r][3], ya.w, u);
            u = dp4(w[r][4], yb.x, u); u = dp4(w[r][5], yb.y, u); u = dp4(w[r][6], yb.z, u); u = dp4(w[r][7], yb.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + blk;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += d[r] * dd * (float(s) + float(u) * kInv254);
            }
        }
    }
}

// ---- TQ2_0: 66 B = qs[64], d (f16) at 64 (quant.py:417-421).  Value 128n + 32g + m is bits 2g of
// byte 32n + m; the code 0..3 stands for code - 1.  Lane q (n = q/4, j = q%4) takes bytes
// 32n + 8j..+7: values m = 8j..8j+7 of all four groups of half n.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_tq2_0(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                           const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int n = q >> 2, j = q & 3;
    uint2 c[RW];
    float d[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 66;
        c[r] = ldw8_a2(b + 32 * n + 8 * j);
        d[r] = h2f(ldw2(b + 64));
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 128 * n + 8 * j;
        const long long g0 = ((tk.tb[t] + (long long)sb * 256) >> 5) + 4 * n;
        int2 xa[4], ya[4];
        float dd[4], ss[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            xa[g] = ldx8(P.xq + o + 32 * g);
            ya[g] = ldx8(P.xq2 + o + 32 * g);
            dd[g] = __ldg(P.xd + g0 + g);
            ss[g] = j == 0 ? __ldg(P.xs + g0 + g) : 0.f;     // the -1 offset once per 32-value group
        }
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            float a = 0.f;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                const uint32_t c0 = (c[r].x >> (2 * g)) & 0x03030303u, c1 = (c[r].y >> (2 * g)) & 0x03030303u;
                const int s = dp4(c1, xa[g].y, dp4(c0, xa[g].x, 0));
                const int u = dp4(c1, ya[g].y, dp4(c0, ya[g].x, 0));
                if constexpr (SUMS) {
                    const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + 4 * n + g;
                    atomicAdd(P.s + base, s);
                    atomicAdd(P.s2 + base, u);
                } else {
                    a += dd[g] * (float(s) + float(u) * kInv254) - ss[g];
                }
            }
            if constexpr (!SUMS) acc[r][t] += d[r] * a;
        }
    }
}

// ---- IQ2_XXS: 66 B = d (f16), 8 x 8 B: per 32 values four codebook indices (u8) and a u32 with four
// 7-bit sign patterns (parity gives the 8th sign) and a 4-bit scale (quant.py:235-245).  Lane q takes
// sub-block q.  The codebook lives in shared memory as (lo, hi) words of eight magnitudes.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_iq2xxs(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                            const Tok<T>& tk, float (&acc)[RW][T], int row0,
                                            const uint2* __restrict__ grid) {
    uint32_t w[RW][8];
    float sc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 66;
        const uint2 a = ldw8_a2(b + 2 + 8 * q);
        sc[r] = h2f(ldw2(b)) * (0.125f + 0.25f * float(a.y >> 28));
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint2 g = grid[(a.x >> (8 * l)) & 0xFFu];
            const uint32_t s7 = (a.y >> (7 * l)) & 127u;
            const uint32_t s8 = s7 | (uint32_t(__popc(s7) & 1) << 7);
            // sign bit k -> byte mask 0xFF at byte k (four bits per word)
            const uint32_t mlo = (((s8 & 15u) * 0x00204081u) & 0x01010101u) * 0xFFu;
            const uint32_t mhi = (((s8 >> 4) * 0x00204081u) & 0x01010101u) * 0xFFu;
            w[r][2 * l] = __vsub4(g.x ^ mlo, mlo);
            w[r][2 * l + 1] = __vsub4(g.y ^ mhi, mhi);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], x0.x, 0); s = dp4(w[r][1], x0.y, s); s = dp4(w[r][2], x0.z, s); s = dp4(w[r][3], x0.w, s);
            s = dp4(w[r][4], x1.x, s); s = dp4(w[r][5], x1.y, s); s = dp4(w[r][6], x1.z, s); s = dp4(w[r][7], x1.w, s);
            int u = dp4(w[r][0], y0.x, 0); u = dp4(w[r][1], y0.y, u); u = dp4(w[r][2], y0.z, u); u = dp4(w[r][3], y0.w, u);
            u = dp4(w[r][4], y1.x, u); u = dp4(w[r][5], y1.y, u); u = dp4(w[r][6], y1.z, u); u = dp4(w[r][7], y1.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + q;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += sc[r] * dd * (float(s) + float(u) * kInv254);
            }
        }
    }
}

// ---- IQ4_XS: 136 B = d (f16), scales_h (u16), scales_l[4], qs[128] (quant.py:378-387).  Lane q takes
// sub-block q: 6-bit scale = nibble q%2 of scales_l[q/2] | bits 2q..2q+1 of scales_h << 4, weight
// scale d * (scale - 32); byte j of qs[16q..] holds codebook indices of values j (low) and 16 + j.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_iq4xs(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                           const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    uint32_t w[RW][8];
    float sc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 136;
        const uint32_t sh = ldw2(b + 2), sl = ldw1(b + 4 + (q >> 1));
        const int ls = int(((sl >> (4 * (q & 1))) & 15u) | (((sh >> (2 * q)) & 3u) << 4));
        sc[r] = h2f(ldw2(b)) * float(ls - 32);
        const uint4 v = ldw16_a2(b + 8 + 16 * q);
        const uint32_t V[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[r][i] = iq4nl_bytes(V[i] & 0x0F0F0F0Fu);
            w[r][4 + i] = iq4nl_bytes((V[i] >> 4) & 0x0F0F0F0Fu);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], x0.x, 0); s = dp4(w[r][1], x0.y, s); s = dp4(w[r][2], x0.z, s); s = dp4(w[r][3], x0.w, s);
            s = dp4(w[r][4], x1.x, s); s = dp4(w[r][5], x1.y, s); s = dp4(w[r][6], x1.z, s); s = dp4(w[r][7], x1.w, s);
            int u = dp4(w[r][0], y0.x, 0); u = dp4(w[r][1], y0.y, u); u = dp4(w[r][2], y0.z, u); u = dp4(w[r][3], y0.w, u);
            u = dp4(w[r][4], y1.x, u); u = dp4(w[r][5], y1.y, u); u = dp4(w[r][6], y1.z, u); u = dp4(w[r][7], y1.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + q;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += sc[r] * dd * (float(s) + float(u) * kInv254);
            }
        }
    }
}

// ---- MXFP4: 17 B = e (E8M0 scale 2^(e-128)), 16 B: byte j holds codebook indices of values j (low
// nibble) and 16 + j (quant.py:390-401).  Lane q takes block 8*sb + q of the row; blocks start at any byte.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_mxfp4(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                           const Tok<T>& tk, float (&acc)[RW][T], int row0) {
    const int blk = sb * 8 + q;
    if (blk >= P.n_in / 32) return;
    uint32_t lo[RW][4], hi[RW][4];
    float d[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)blk * 17;
        d[r] = mxfp4_scale(ldw1(b));
        const uint4 v = ldw16_a1(b + 1);
        const uint32_t V[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo[r][i] = mxfp4_bytes(V[i] & 0x0F0F0F0Fu);
            hi[r][i] = mxfp4_bytes((V[i] >> 4) & 0x0F0F0F0Fu);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)blk * 32;
        const int4 xa = ldx16(P.xq + o), xb = ldx16(P.xq + o + 16);
        const int4 ya = ldx16(P.xq2 + o), yb = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + (tk.tb[t] >> 5) + blk);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(lo[r][0], xa.x, 0); s = dp4(lo[r][1], xa.y, s); s = dp4(lo[r][2], xa.z, s); s = dp4(lo[r][3], xa.w, s);
            s = dp4(hi[r][0], xb.x, s); s = dp4(hi[r][1], xb.y, s); s = dp4(hi[r][2], xb.z, s); s = dp4(hi[r][3], xb.w, s);
            int u = dp4(lo[r][0], ya.x, 0); u = dp4(lo[r][1], ya.y, u); u = dp4(lo[r][2], ya.z, u); u = dp4(lo[r][3], ya.w, u);
            u = dp4(hi[r][0], yb.x, u); u = dp4(hi[r][1], yb.y, u); u = dp4(hi[r][2], yb.z, u); u = dp4(hi[r][3], yb.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + blk;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += d[r] * dd * (float(s) + float(u) * kInv254);
            }
        }
    }
}

// ---- IQ3_S: 110 B = d (f16), qs[64], qh[8], signs[32], scales[4] (quant.py:334-346).  Lane q takes
// sub-block q: group l (4 values) has codebook index qs[8q + l] | bit l of qh[q] << 8 and the signs in
// bits 4l..4l+3 of the sub-block's four sign bytes; weight scale d * (1 + 2 * 4-bit scale).  The 512
// entries sit in shared memory as four magnitude bytes each.
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_iq3s(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                          const Tok<T>& tk, float (&acc)[RW][T], int row0,
                                          const uint32_t* __restrict__ grid) {
    uint32_t w[RW][8];
    float sc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 110;
        const uint2 qs = ldw8_a2(b + 2 + 8 * q);
        const uint32_t qh = ldw1(b + 66 + q);
        const uint32_t sg = ldw2(b + 74 + 4 * q) | (ldw2(b + 76 + 4 * q) << 16);
        const uint32_t ls = (ldw1(b + 106 + (q >> 1)) >> (4 * (q & 1))) & 15u;
        sc[r] = h2f(ldw2(b)) * float(1 + 2 * int(ls));
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t idx = (((l < 4 ? qs.x : qs.y) >> (8 * (l & 3))) & 0xFFu) | (((qh >> l) & 1u) << 8);
            const uint32_t m = sign4_mask(sg >> (4 * l));
            w[r][l] = __vsub4(grid[idx] ^ m, m);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], x0.x, 0); s = dp4(w[r][1], x0.y, s); s = dp4(w[r][2], x0.z, s); s = dp4(w[r][3], x0.w, s);
            s = dp4(w[r][4], x1.x, s); s = dp4(w[r][5], x1.y, s); s = dp4(w[r][6], x1.z, s); s = dp4(w[r][7], x1.w, s);
            int u = dp4(w[r][0], y0.x, 0); u = dp4(w[r][1], y0.y, u); u = dp4(w[r][2], y0.z, u); u = dp4(w[r][3], y0.w, u);
            u = dp4(w[r][4], y1.x, u); u = dp4(w[r][5], y1.y, u); u = dp4(w[r][6], y1.z, u); u = dp4(w[r][7], y1.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + q;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += sc[r] * dd * (float(s) + float(u) * kInv254);
            }
        }
    }
}

// ---- IQ3_XXS: 98 B = d (f16), qs[64], aux u32[8] (quant.py:322-331).  Lane q takes sub-block q: values
// 4k..4k+3 are codebook entry qs[8q + k]; aux[q] holds four 7-bit sign groups of 8 values (parity gives
// the 8th sign) and the 4-bit scale s in bits 28..31: weight scale d * (0.25 + 0.5 s).
template <int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_iq3xxs(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                            const Tok<T>& tk, float (&acc)[RW][T], int row0,
                                            const uint32_t* __restrict__ grid) {
    uint32_t w[RW][8];
    float sc[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
        const uint8_t* b = rows[r] + (long long)sb * 98;
        const uint2 qs = ldw8_a2(b + 2 + 8 * q);
        const uint32_t aux = ldw2(b + 66 + 4 * q) | (ldw2(b + 68 + 4 * q) << 16);
        sc[r] = h2f(ldw2(b)) * (0.25f + 0.5f * float(aux >> 28));
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const uint32_t s7 = (aux >> (7 * l)) & 127u;
            const uint32_t s8 = s7 | (uint32_t(__popc(s7) & 1) << 7);
            const uint32_t mlo = sign4_mask(s8), mhi = sign4_mask(s8 >> 4);
            const uint32_t word = l < 2 ? qs.x : qs.y;
            w[r][2 * l] = __vsub4(grid[(word >> (16 * (l & 1))) & 0xFFu] ^ mlo, mlo);
            w[r][2 * l + 1] = __vsub4(grid[(word >> (16 * (l & 1) + 8)) & 0xFFu] ^ mhi, mhi);
        }
    }
#pragma unroll
    for (int t = 0; t < T; ++t) {
        const long long o = tk.tb[t] + (long long)sb * 256 + 32 * q;
        const int4 x0 = ldx16(P.xq + o), x1 = ldx16(P.xq + o + 16);
        const int4 y0 = ldx16(P.xq2 + o), y1 = ldx16(P.xq2 + o + 16);
        const float dd = __ldg(P.xd + ((tk.tb[t] + (long long)sb * 256) >> 5) + q);
#pragma unroll
        for (int r = 0; r < RW; ++r) {
            int s = dp4(w[r][0], x0.x, 0); s = dp4(w[r][1], x0.y, s); s = dp4(w[r][2], x0.z, s); s = dp4(w[r][3], x0.w, s);
            s = dp4(w[r][4], x1.x, s); s = dp4(w[r][5], x1.y, s); s = dp4(w[r][6], x1.z, s); s = dp4(w[r][7], x1.w, s);
            int u = dp4(w[r][0], y0.x, 0); u = dp4(w[r][1], y0.y, u); u = dp4(w[r][2], y0.z, u); u = dp4(w[r][3], y0.w, u);
            u = dp4(w[r][4], y1.x, u); u = dp4(w[r][5], y1.y, u); u = dp4(w[r][6], y1.z, u); u = dp4(w[r][7], y1.w, u);
            if constexpr (SUMS) {
                const long long base = (long long)row0 * (P.n_in / 32) + sb * 8 + q;
                atomicAdd(P.s + base, s);
                atomicAdd(P.s2 + base, u);
            } else {
                acc[r][t] += sc[r] * dd * (float(s) + float(u) * kInv254);
            }
        }
    }
}

// IQ3_XXS codebook, 3 bits per magnitude (index into {4, 12, 20, 28, 36, 44, 52, 62})
__device__ const uint16_t kIq3xxsCodes[256] = {
#include "iq3xxs_grid.inc"
};

__device__ __forceinline__ void load_iq3xxs_grid(uint32_t* grid) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        const uint32_t c = kIq3xxsCodes[i];
        uint32_t w = 0u;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t lv = (c >> (3 * k)) & 7u;
            w |= (lv == 7u ? 62u : 4u + 8u * lv) << (8 * k);
        }
        grid[i] = w;
    }
}

// IQ3_S codebook, 3 bits per magnitude ((m - 1) / 2); expanded per block at launch
__device__ const uint16_t kIq3sCodes[512] = {
#include "iq3s_grid.inc"
};

__device__ __forceinline__ void load_iq3s_grid(uint32_t* grid) {
    for (int i = threadIdx.x; i < 512; i += blockDim.x) {
        const uint32_t c = kIq3sCodes[i];
        uint32_t w = 0u;
#pragma unroll
        for (int k = 0; k < 4; ++k) w |= (2u * ((c >> (3 * k)) & 7u) + 1u) << (8 * k);
        grid[i] = w;
    }
}

// IQ2_XXS codebook, 2 bits per magnitude (index into {8, 25, 43}); expanded per block at launch
__device__ const uint16_t kIq2xxsCodes[256] = {
#include "iq2xxs_grid.inc"
};

__device__ __forceinline__ void load_iq2xxs_grid(uint2* grid) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) {
        const uint32_t c = kIq2xxsCodes[i];
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t lv = (c >> (2 * k)) & 3u;
            const uint32_t mag = lv == 0 ? 8u : (lv == 1 ? 25u : 43u);
            w[k >> 2] |= mag << (8 * (k & 3));
        }
        grid[i] = make_uint2(w[0], w[1]);
    }
}

// Weight row base of slot `slot`: the dense matrix, expert ids[slot] of a packed expert tensor, or an
// address-table entry.  Returns nullptr (and flags the status word) for an address that the
// format's loads cannot use.
template <int FMT>
__device__ __forceinline__ const uint8_t* slot_base(const MvParams& P, int slot) {
    if (P.ids == nullptr) return P.w;
    const long long e = P.ids[slot];
    if (e < 0 || e >= P.n_exp) {
        // -1 marks an unused slot (a padded exchange buffer): zeros, no error
        if (e != kPadSlot && P.status) atomicOr(P.status, DEV_BAD_ADDRESS);
        return nullptr;
    }
    const uint8_t* base = P.per_expert >= 0 ? P.w + e * P.per_expert
                                            : reinterpret_cast<const uint8_t*>(reinterpret_cast<const long long*>(P.w)[e]);
    const uintptr_t need = uintptr_t(weight_align(FMT) - 1);
    if (reinterpret_cast<uintptr_t>(base) & need) {
        if (P.status) atomicOr(P.status, DEV_BAD_ADDRESS);
        return nullptr;
    }
    return base;
}

// codebook of the formats that keep one in shared memory (2 KB), loaded by the whole block
template <int FMT>
__host__ __device__ constexpr bool smem_grid_format() { return FMT == F_IQ2_XXS || FMT == F_IQ3_S || FMT == F_IQ3_XXS; }
template <int FMT>
__device__ __forceinline__ void load_grid(uint2* grid) {
    if constexpr (FMT == F_IQ2_XXS) load_iq2xxs_grid(grid);
    else if constexpr (FMT == F_IQ3_S) load_iq3s_grid(reinterpret_cast<uint32_t*>(grid));
    else if constexpr (FMT == F_IQ3_XXS) load_iq3xxs_grid(reinterpret_cast<uint32_t*>(grid));
}

// One lane's part of 256-value piece sb of RW rows for T tokens (the lane layout above), any format.
template <int FMT, int T, int RW, bool SUMS>
__device__ __forceinline__ void lane_any(const uint8_t* const (&rows)[RW], int sb, int q, const MvParams& P,
                                         const Tok<T>& tk, float (&acc)[RW][T], int row0, const uint2* grid) {
    if constexpr (FMT == F_Q4_K) lane_q4k<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_Q5_K) lane_q4k<T, RW, SUMS, true>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_Q6_K) lane_q6k<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_Q4_0) lane_q4_0<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_Q8_0) lane_q8_0<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_TQ2_0) lane_tq2_0<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_IQ4_XS) lane_iq4xs<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_MXFP4) lane_mxfp4<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_IQ3_S)
        lane_iq3s<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0, reinterpret_cast<const uint32_t*>(grid));
    else if constexpr (FMT == F_IQ3_XXS)
        lane_iq3xxs<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0, reinterpret_cast<const uint32_t*>(grid));
    else if constexpr (FMT == F_Q4_1 || FMT == F_Q5_0 || FMT == F_Q5_1 || FMT == F_IQ4_NL)
        lane_b32<FMT, T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (bits_format(FMT)) lane_bits<T, RW, SUMS, FMT>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_Q3_K) lane_q3k<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (iq2x_format(FMT)) lane_iq2x<T, RW, SUMS, FMT>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_Q2_K) lane_q2k<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_TQ1_0) lane_tq1<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (iq1_format(FMT)) lane_iq1<T, RW, SUMS, FMT>(rows, sb, q, P, tk, acc, row0);
    else if constexpr (FMT == F_PTQ1_0) lane_ptq1<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0);
    else lane_iq2xxs<T, RW, SUMS>(rows, sb, q, P, tk, acc, row0, grid);
}

// y[slot][t][row] = W_slot[row, :] . x(slot, t) for T tokens.  Each warp takes RW consecutive rows
// of one slot at a time (grid-stride over all slots' row groups); SUMS instead adds the int32 unit
// sums of one token into P.s / P.s2 (T = RW = 1).
template <int FMT, int T, int RW, bool SUMS>
__global__ void __launch_bounds__(256) mv_kernel(const MvParams P) {
    __shared__ uint2 grid[smem_grid_format<FMT>() ? 256 : 1];   // 2 KB: a codebook
    if constexpr (smem_grid_format<FMT>()) {
        load_grid<FMT>(grid);
        __syncthreads();
    }
    const int lane = threadIdx.x & 31, q = lane & 7, sb0 = lane >> 3;
    const int groups = (P.n_out + RW - 1) / RW;
    const long long total = (long long)groups * P.slots;
    const long long warps = (long long)gridDim.x * kWarpsPerBlock;
    const int n_sb = (P.n_in + 255) >> 8;                 // 256-value pieces (8 blocks of 32-value formats)
    for (long long it = (long long)blockIdx.x * kWarpsPerBlock + (threadIdx.x >> 5); it < total; it += warps) {
        const int slot = int(it / groups);
        const int row0 = int(it % groups) * RW;
        const uint8_t* base = slot_base<FMT>(P, slot);
        if (base == nullptr) {                            // refused slot (whole warp): defined zeros
            if (!SUMS && lane < RW * T) {
                const int r = lane / T, t = lane % T;
                if (row0 + r < P.n_out) P.y[((long long)slot * T + t) * P.n_out + row0 + r] = 0.f;
            }
            continue;
        }
        const uint8_t* rows[RW];
#pragma unroll
        for (int r = 0; r < RW; ++r) rows[r] = base + (long long)min(row0 + r, P.n_out - 1) * P.row_bytes;
        Tok<T> tk;
#pragma unroll
        for (int t = 0; t < T; ++t) tk.tb[t] = (long long)(slot / P.x_group + t) * P.n_in;
        float acc[RW][T];
#pragma unroll
        for (int r = 0; r < RW; ++r)
#pragma unroll
            for (int t = 0; t < T; ++t) acc[r][t] = 0.f;
        for (int sb = sb0; sb < n_sb; sb += 4) lane_any<FMT, T, RW, SUMS>(rows, sb, q, P, tk, acc, row0, grid);
        if constexpr (!SUMS) {
#pragma unroll
            for (int r = 0; r < RW; ++r)
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    const float v = warp_sum(acc[r][t]);
                    if (lane == 0 && row0 + r < P.n_out)
                        P.y[((long long)slot * T + t) * P.n_out + row0 + r] = v;
                }
        }
    }
}

}  // namespace qmv
