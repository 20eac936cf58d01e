// Few-token matvec (2..8 tokens) for Q4_K rows on the tensor cores: y[t] = W x_t.
//
// The weights stream through the same bulk-copy ring as the single-token kernel, in tiles of 16 rows
// (one MMA row block), one copy per row into rows padded by 16 bytes: the eight rows of an A fragment
// then fall on distinct banks (unpadded Q4_K rows are a multiple of 128 bytes apart).  The tokens' two-stage int8 activations sit in shared memory (token rows padded
// by 16 bytes, so the eight tokens of a B fragment fall on distinct banks).  Each consumer warp takes
// whole superblocks of every tile: per 32-value sub-block it forms the A fragment from the nibbles in
// shared memory (codes 0..15, unsigned), runs two mma.sync.m16n8k32 (tokens' xq and xq2 as B; N = 8
// tokens, unused tokens zero), and scales the int32 sums in registers:
//     y[r][t] += d_r sc_rj * (xd_tj / 254) * (254 S + S2) - dmin_r m_rj * xs_tj
// the same integer sums and epilogue terms as the single-token path (ggufengine/mmvq.py:389-404 per
// token).  Per-sub-block scales are why the accumulators live in registers: a tensor-memory
// accumulator would have to be read back after every K = 32 step.  Warps' partial sums meet in shared
// memory and are added in a fixed order.  Every mbarrier wait is bounded.
#pragma once
#include "qmv_tma.cuh"

namespace qmv {

constexpr int kMmaRows = 16;                     // rows per tile (the MMA's M)
constexpr int kMmaMaxTok = 8;                    // the MMA's N
constexpr int kMmaMaxIn = 4096;                  // activation rows staged in shared memory

struct MmaParams {
    const uint8_t* w;
    float* y;                                    // [token][n_out]
    const int8_t* xq;                            // [token][n_in] (Eingang layout)
    const int8_t* xq2;
    const float* xd;                             // [token][n_in / 32]
    const float* xs;
    long long row_bytes;
    int n_out, n_in, n_tok, stages;
    int* status;
};

__host__ __device__ constexpr int mma_act_stride(int n_in) { return n_in + 16; }
__host__ __device__ constexpr int mma_scale_stride(int n_in) { return n_in / 32 + 4; }   // floats per token
__host__ __device__ constexpr long long mma_row_stride(long long row_bytes) { return row_bytes + 16; }
__host__ __device__ constexpr long long mma_act_bytes(int n_in) {
    return 2LL * kMmaMaxTok * mma_act_stride(n_in) + 2LL * kMmaMaxTok * mma_scale_stride(n_in) * 4;
}
__host__ __device__ constexpr int mma_red_bytes(int ncw) { return ncw * kMmaRows * kMmaMaxTok * 4; }

// D = A (16x32 u8) * B (32x8 s8) + D, int32
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 6-bit scales and mins of the 8 sub-blocks of a Q4_K superblock (header words y, z, w), one per byte
__device__ __forceinline__ void q4k_scale_words(uint4 hd, uint32_t& sc_lo, uint32_t& sc_hi, uint32_t& m_lo, uint32_t& m_hi) {
    sc_lo = hd.y & 0x3F3F3F3Fu;
    m_lo = hd.z & 0x3F3F3F3Fu;
    sc_hi = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
    m_hi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
}

template <int NCW>
__global__ void __launch_bounds__(32 * (NCW + 1), 1) mv_mma_q4k_kernel(const MmaParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = P.stages;
    const uint32_t rstride = uint32_t(mma_row_stride(P.row_bytes));
    const uint32_t slot_bytes = kMmaRows * rstride;
    const int stride = mma_act_stride(P.n_in), ng = P.n_in / 32, gs = mma_scale_stride(P.n_in);
    int8_t* aq = reinterpret_cast<int8_t*>(smem + (long long)S * slot_bytes);
    int8_t* aq2 = aq + kMmaMaxTok * stride;
    float* ad = reinterpret_cast<float*>(aq2 + kMmaMaxTok * stride);
    float* as = ad + kMmaMaxTok * gs;
    float* red = as + kMmaMaxTok * gs;
    uint64_t* bars = reinterpret_cast<uint64_t*>(red + NCW * kMmaRows * kMmaMaxTok);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S), stage0 = smem_u32(smem);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_tiles = (P.n_out + kMmaRows - 1) / kMmaRows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, NCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer: 16-row tiles t = blockIdx.x, + grid, ... ----------------
        if (lane != 0) return;
        int it = 0;
        bool ok = true;
        for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
            const int s = it % S;
            if (it >= S && !mbar_wait(empty0 + 8 * s, ((it / S) & 1) ^ 1)) {
                ok = false;
                break;
            }
            const int r0 = t * kMmaRows, nr = min(kMmaRows, P.n_out - r0);
            mbar_arrive_tx(full0 + 8 * s, uint32_t(nr * P.row_bytes));
            for (int r = 0; r < nr; ++r)
                bulk_g2s(stage0 + uint32_t(s) * slot_bytes + uint32_t(r) * rstride, P.w + (long long)(r0 + r) * P.row_bytes,
                         uint32_t(P.row_bytes), full0 + 8 * s);
        }
        if (!ok) {
            if (P.status) atomicOr(P.status, DEV_TIMEOUT);
            for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(full0 + 8 * (k % S), (k / S) & 1);
        }
        return;
    }

    // ---------------- consumers ----------------
    // the tokens' activations (tokens >= n_tok: zeros) into shared memory
    const int cl = threadIdx.x, nthr = 32 * NCW;
    for (int i = cl; i < kMmaMaxTok * (P.n_in / 16); i += nthr) {
        const int t = i / (P.n_in / 16), c = i % (P.n_in / 16);
        int4 a = make_int4(0, 0, 0, 0), b = a;
        if (t < P.n_tok) {
            a = __ldg(reinterpret_cast<const int4*>(P.xq + (long long)t * P.n_in) + c);
            b = __ldg(reinterpret_cast<const int4*>(P.xq2 + (long long)t * P.n_in) + c);
        }
        *reinterpret_cast<int4*>(aq + t * stride + 16 * c) = a;
        *reinterpret_cast<int4*>(aq2 + t * stride + 16 * c) = b;
    }
    for (int i = cl; i < kMmaMaxTok * ng; i += nthr) {
        const int t = i / ng, g = i % ng;
        ad[t * gs + g] = t < P.n_tok ? __ldg(P.xd + (long long)t * ng + g) * kInv254 : 0.f;
        as[t * gs + g] = t < P.n_tok ? __ldg(P.xs + (long long)t * ng + g) : 0.f;
    }
    named_sync(kConsumerBarrier, nthr);

    const int gid = lane >> 2, tig = lane & 3;            // MMA fragment coordinates
    const int n_sb = P.n_in / 256;
    bool dead = false;
    int it = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++it) {
        const int s = it % S;
        const bool got = !dead && mbar_wait(full0 + 8 * s, (it / S) & 1);
        if (!got && !dead) {
            dead = true;
            if (lane == 0 && P.status) atomicOr(P.status, DEV_TIMEOUT);
        }
        const uint32_t tile = stage0 + uint32_t(s) * slot_bytes;
        // rows gid and gid + 8 of the tile x tokens 2 tig, 2 tig + 1
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        if (got) {
            const uint32_t rg = tile + uint32_t(gid) * rstride, rh = tile + uint32_t(gid + 8) * rstride;
            for (int sb = warp; sb < n_sb; sb += NCW) {
                const uint32_t bg = rg + sb * 144, bh = rh + sb * 144;
                const uint4 hg = lds128(bg), hh = lds128(bh);
                uint32_t scg_lo, scg_hi, mg_lo, mg_hi, sch_lo, sch_hi, mh_lo, mh_hi;
                q4k_scale_words(hg, scg_lo, scg_hi, mg_lo, mg_hi);
                q4k_scale_words(hh, sch_lo, sch_hi, mh_lo, mh_hi);
                const float dg = h2f(hg.x & 0xFFFFu), dmg = h2f(hg.x >> 16);
                const float dh = h2f(hh.x & 0xFFFFu), dmh = h2f(hh.x >> 16);
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    // k = 4 tig .. and 16 + 4 tig .. of the 32 bytes of pair p (low nibbles: sub-block 2p)
                    const uint32_t wg0 = lds32(bg + 16 + 32 * p + 4 * tig), wg1 = lds32(bg + 32 + 32 * p + 4 * tig);
                    const uint32_t wh0 = lds32(bh + 16 + 32 * p + 4 * tig), wh1 = lds32(bh + 32 + 32 * p + 4 * tig);
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        const int j = 2 * p + half, sh = 4 * half;
                        const uint32_t a0 = (wg0 >> sh) & 0x0F0F0F0Fu, a1 = (wh0 >> sh) & 0x0F0F0F0Fu;
                        const uint32_t a2 = (wg1 >> sh) & 0x0F0F0F0Fu, a3 = (wh1 >> sh) & 0x0F0F0F0Fu;
                        const int k0 = 256 * sb + 32 * j + 4 * tig;           // value index of b0 (token gid)
                        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(aq + gid * stride + k0);
                        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(aq + gid * stride + k0 + 16);
                        const uint32_t c0 = *reinterpret_cast<const uint32_t*>(aq2 + gid * stride + k0);
                        const uint32_t c1 = *reinterpret_cast<const uint32_t*>(aq2 + gid * stride + k0 + 16);
                        int s1[4] = {0, 0, 0, 0}, s2[4] = {0, 0, 0, 0};
                        mma_u8s8(s1, a0, a1, a2, a3, b0, b1);
                        mma_u8s8(s2, a0, a1, a2, a3, c0, c1);
                        // scales of sub-block j: byte j % 4 of the low (j < 4) or high words
                        const int bsh = 8 * (j & 3);
                        const float wsg = dg * float(((j < 4 ? scg_lo : scg_hi) >> bsh) & 0xFFu);
                        const float msg = dmg * float(((j < 4 ? mg_lo : mg_hi) >> bsh) & 0xFFu);
                        const float wsh = dh * float(((j < 4 ? sch_lo : sch_hi) >> bsh) & 0xFFu);
                        const float msh = dmh * float(((j < 4 ? mh_lo : mh_hi) >> bsh) & 0xFFu);
                        const int blk = 8 * sb + j;
                        const float xd0 = ad[(2 * tig) * gs + blk], xd1 = ad[(2 * tig + 1) * gs + blk];
                        const float xs0 = as[(2 * tig) * gs + blk], xs1 = as[(2 * tig + 1) * gs + blk];
                        acc[0] += wsg * xd0 * float(254 * s1[0] + s2[0]) - msg * xs0;
                        acc[1] += wsg * xd1 * float(254 * s1[1] + s2[1]) - msg * xs1;
                        acc[2] += wsh * xd0 * float(254 * s1[2] + s2[2]) - msh * xs0;
                        acc[3] += wsh * xd1 * float(254 * s1[3] + s2[3]) - msh * xs1;
                    }
                }
            }
        }
        __syncwarp();
        if (got && lane == 0) mbar_arrive(empty0 + 8 * s);
        // partial sums of this warp's superblocks: [warp][row][token]
        float* rw = red + warp * kMmaRows * kMmaMaxTok;
        rw[gid * kMmaMaxTok + 2 * tig] = acc[0];
        rw[gid * kMmaMaxTok + 2 * tig + 1] = acc[1];
        rw[(gid + 8) * kMmaMaxTok + 2 * tig] = acc[2];
        rw[(gid + 8) * kMmaMaxTok + 2 * tig + 1] = acc[3];
        named_sync(kConsumerBarrier, nthr);
        if (cl < kMmaRows * kMmaMaxTok && !dead) {
            const int r = cl / kMmaMaxTok, tk = cl % kMmaMaxTok, row = t * kMmaRows + r;
            float v = 0.f;
            for (int w = 0; w < NCW; ++w) v += red[w * kMmaRows * kMmaMaxTok + cl];   // fixed order
            if (tk < P.n_tok && row < P.n_out) P.y[(long long)tk * P.n_out + row] = v;
        }
        named_sync(kConsumerBarrier, nthr);
    }
}

}  // namespace qmv
