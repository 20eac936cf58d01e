// Few-token matvec (2..8 tokens) for Q4_K and Q8_0 rows on the tensor cores: y[t] = W x_t.
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
// Q8_0 (34-byte blocks: d, 32 int8): each warp takes whole blocks; A = the int8 codes (2-byte aligned
// in shared memory: aligned words and funnel shifts), two mma.sync.m16n8k32 s8 x s8 per block and
//     y[r][t] += d_r * (xd_t / 254) * (254 S + S2).
#pragma once
#include "qmv_tma.cuh"

namespace qmv {

constexpr int kMmaRows = 16;                     // rows per tile (the MMA's M)
constexpr int kMmaMaxTok = 8;                    // the MMA's N
constexpr int kMmaMaxIn = 4096;                  // activation rows staged in shared memory

constexpr int kMmaJobs = 4;                       // matrices of one mv_mma_kernel launch (same input)

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
    // mv_mma_kernel: jobs j < n_jobs (matrices reading the same tokens), weights jw[j], outputs jy[j]
    // ([token][jn[j]]), 16-row tiles jt[j] .. jt[j + 1] - 1 of the launch's tile list
    int n_jobs;
    const uint8_t* jw[kMmaJobs];
    float* jy[kMmaJobs];
    int jn[kMmaJobs];
    int jt[kMmaJobs + 1];
};

struct MmaTile {
    const uint8_t* w;
    float* y;
    int r0, nr, n_out;
};
// tile t of the launch: its job's weights and outputs, first row and rows
__device__ __forceinline__ MmaTile mma_tile(const MmaParams& P, int t) {
    int j = 0;
    while (j + 1 < P.n_jobs && t >= P.jt[j + 1]) ++j;
    MmaTile m;
    m.w = P.jw[j];
    m.y = P.jy[j];
    m.n_out = P.jn[j];
    m.r0 = (t - P.jt[j]) * kMmaRows;
    m.nr = min(kMmaRows, m.n_out - m.r0);
    return m;
}

__host__ __device__ constexpr int mma_act_stride(int n_in) { return n_in + 16; }
__host__ __device__ constexpr int mma_scale_stride(int n_in) { return n_in / 32 + 4; }   // floats per token
__host__ __device__ constexpr long long mma_row_stride(long long row_bytes) { return row_bytes + 16; }
__host__ __device__ constexpr long long mma_act_bytes(int n_in) {
    return 2LL * kMmaMaxTok * mma_act_stride(n_in) + 2LL * kMmaMaxTok * mma_scale_stride(n_in) * 4;
}
__host__ __device__ constexpr int mma_red_bytes(int ncw) { return ncw * kMmaRows * kMmaMaxTok * 4; }

// 4 bytes at a 2-byte aligned shared address
__device__ __forceinline__ uint32_t lds32_a2(uint32_t a) {
    const uint32_t b = a & ~3u, sh = (a & 3u) * 8u;
    return __funnelshift_r(lds32(b), lds32(b + 4), sh);
}

// D = A (16x32 s8) * B (32x8 s8) + D, int32
__device__ __forceinline__ void mma_s8s8_k32(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                             uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
                 "{%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

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

template <int FMT, int NCW>
__global__ void __launch_bounds__(32 * (NCW + 1), 1) mv_mma_kernel(const MmaParams P) {
    static_assert(FMT == F_Q4_K || FMT == F_Q8_0, "few-token tensor-core formats");
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
    const int n_tiles = P.jt[P.n_jobs];
    // programmatic dependent launch: the next kernel may launch now (its weight copies do not read our
    // outputs); the consumers read the activation only after the previous kernel has completed
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

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
            const MmaTile m = mma_tile(P, t);
            mbar_arrive_tx(full0 + 8 * s, uint32_t(m.nr * P.row_bytes));
            for (int r = 0; r < m.nr; ++r)
                bulk_g2s(stage0 + uint32_t(s) * slot_bytes + uint32_t(r) * rstride, m.w + (long long)(m.r0 + r) * P.row_bytes,
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
    asm volatile("griddepcontrol.wait;" ::: "memory");
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
        if (got && FMT == F_Q8_0) {
            const uint32_t rg = tile + uint32_t(gid) * rstride, rh = tile + uint32_t(gid + 8) * rstride;
            for (int blk = warp; blk < ng; blk += NCW) {
                const uint32_t bg = rg + blk * 34, bh = rh + blk * 34;
                // k = 4 tig .. and 16 + 4 tig .. of the block's 32 codes (rows gid, gid + 8)
                const uint32_t a0 = lds32_a2(bg + 2 + 4 * tig), a1 = lds32_a2(bh + 2 + 4 * tig);
                const uint32_t a2 = lds32_a2(bg + 18 + 4 * tig), a3 = lds32_a2(bh + 18 + 4 * tig);
                const int k0 = 32 * blk + 4 * tig;
                const uint32_t b0 = *reinterpret_cast<const uint32_t*>(aq + gid * stride + k0);
                const uint32_t b1 = *reinterpret_cast<const uint32_t*>(aq + gid * stride + k0 + 16);
                const uint32_t c0 = *reinterpret_cast<const uint32_t*>(aq2 + gid * stride + k0);
                const uint32_t c1 = *reinterpret_cast<const uint32_t*>(aq2 + gid * stride + k0 + 16);
                int s1[4] = {0, 0, 0, 0}, s2[4] = {0, 0, 0, 0};
                mma_s8s8_k32(s1, a0, a1, a2, a3, b0, b1);
                mma_s8s8_k32(s2, a0, a1, a2, a3, c0, c1);
                const float dg = h2f(lds16u(bg)), dh = h2f(lds16u(bh));
                const float xd0 = ad[(2 * tig) * gs + blk], xd1 = ad[(2 * tig + 1) * gs + blk];
                acc[0] += dg * xd0 * float(254 * s1[0] + s2[0]);
                acc[1] += dg * xd1 * float(254 * s1[1] + s2[1]);
                acc[2] += dh * xd0 * float(254 * s1[2] + s2[2]);
                acc[3] += dh * xd1 * float(254 * s1[3] + s2[3]);
            }
        } else if (got) {
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
            const MmaTile m = mma_tile(P, t);
            const int r = cl / kMmaMaxTok, tk = cl % kMmaMaxTok, row = m.r0 + r;
            float v = 0.f;
            for (int w = 0; w < NCW; ++w) v += red[w * kMmaRows * kMmaMaxTok + cl];   // fixed order
            if (tk < P.n_tok && r < m.nr) m.y[(long long)tk * m.n_out + row] = v;
        }
        named_sync(kConsumerBarrier, nthr);
    }
}

}  // namespace qmv

namespace qmv {

// ---- few-token Q6_K (rows of any multiple of 2048 values) -----------------------------------------
// Tiles are 16 rows x one 2048-value chunk of K (16 copies of 1680 bytes: eight superblocks per row;
// 1680 = 16 mod 128, so the eight rows of a fragment fall on distinct banks).  A CTA walks its row
// blocks chunk by chunk, K-chunk major, keeping each row block's running sums per (row, token) in
// shared memory (added in chunk order: deterministic).  The activation chunk of every token (xq, xq2
// 2048 bytes each, xd 64 floats) is brought into one of two shared buffers by the producer's bulk
// copies ahead of the chunk's weight tiles (own mbarriers), token rows padded by 16 bytes for
// conflict-free B fragments.  Per 16-value group (one Q6_K scale): A = code - 32 as signed bytes,
// mma.sync.m16n8k16 with xq and with xq2, y[r][t] += d_r sc_rg * (xd_tg / 254) * (254 S + S2).

constexpr int kQ6Chunk = 2048;                     // values per K-chunk
constexpr int kQ6ChunkBytes = kQ6Chunk / 256 * 210;  // 1680
constexpr int kQ6MaxBlocks = 64;                   // row blocks per CTA whose sums fit in shared memory
constexpr int kQ6RegBlocks = 4;                    // row blocks per CTA whose sums stay in registers
constexpr int kQ6ActStride = kQ6Chunk + 16;        // bytes per token row of a staged activation chunk
// one staged chunk: xq [8][stride], xq2 [8][stride], xd [8][64 + 4] floats
constexpr int kQ6ActBytes = 2 * kMmaMaxTok * kQ6ActStride + kMmaMaxTok * (kQ6Chunk / 32 + 4) * 4;

__device__ __forceinline__ void mma_s8s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a0), "r"(a1), "r"(b0));
}
// four unsigned 6-bit codes -> code - 32 as signed bytes (no carries between bytes)
__device__ __forceinline__ uint32_t q6_signed(uint32_t c) {
    return ((c | 0x80808080u) - 0x20202020u) ^ 0x80808080u;
}

template <int NCW>
__global__ void __launch_bounds__(32 * (NCW + 1), 1) mv_mma_q6k_kernel(const MmaParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = P.stages;
    const uint32_t slot_bytes = kMmaRows * kQ6ChunkBytes;
    uint8_t* actb = smem + (long long)S * slot_bytes;                // two staged activation chunks
    float* red = reinterpret_cast<float*>(actb + 2 * kQ6ActBytes);
    float* run = red + NCW * kMmaRows * kMmaMaxTok;                 // [local block][row][token]
    const int n_rb = (P.n_out + kMmaRows - 1) / kMmaRows, n_kc = P.n_in / kQ6Chunk;
    const int my_rb = (n_rb - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
    uint64_t* bars = reinterpret_cast<uint64_t*>(run + kQ6MaxBlocks * kMmaRows * kMmaMaxTok);
    const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + S), stage0 = smem_u32(smem);
    const uint32_t afull0 = smem_u32(bars + 2 * S), aempty0 = smem_u32(bars + 2 * S + 2);
    const int ng = P.n_in / 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // as in mv_mma_kernel

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full0 + 8 * s, 1);
            mbar_init(empty0 + 8 * s, NCW);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(afull0 + 8 * b, 1);
            mbar_init(aempty0 + 8 * b, NCW);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == NCW) {
        // ---------------- producer: per chunk kc its activation, then tiles (kc, rb), rb = blockIdx.x + grid i ----
        if (lane != 0) return;
        int it = 0;
        bool ok = true;
        for (int kc = 0; kc < n_kc && ok; ++kc) {
            const int ab = kc & 1;
            if (kc >= 2 && !mbar_wait(aempty0 + 8 * ab, ((kc / 2) & 1) ^ 1)) {
                ok = false;
                break;
            }
            const uint32_t abuf = smem_u32(actb + ab * kQ6ActBytes);
            auto copy_act = [&]() {
                mbar_arrive_tx(afull0 + 8 * ab, uint32_t(P.n_tok * (2 * kQ6Chunk + 4 * (kQ6Chunk / 32))));
                for (int t = 0; t < P.n_tok; ++t) {
                    const long long o = (long long)t * P.n_in + (long long)kc * kQ6Chunk;
                    bulk_g2s(abuf + t * kQ6ActStride, P.xq + o, kQ6Chunk, afull0 + 8 * ab);
                    bulk_g2s(abuf + (kMmaMaxTok + t) * kQ6ActStride, P.xq2 + o, kQ6Chunk, afull0 + 8 * ab);
                    bulk_g2s(abuf + 2 * kMmaMaxTok * kQ6ActStride + t * (kQ6Chunk / 32 + 4) * 4,
                             P.xd + (long long)t * ng + kc * (kQ6Chunk / 32), 4 * (kQ6Chunk / 32), afull0 + 8 * ab);
                }
            };
            // chunk 0: the first S tiles (no slot to wait for) go out before its activation, which is
            // read only after the previous kernel has completed; later chunks: activation first
            const int pre = kc == 0 ? min(S, my_rb) : 0;
            bool act_sent = false;
            for (int i = 0; i < my_rb; ++i, ++it) {
                if (!act_sent && i >= pre) {
                    if (kc == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
                    copy_act();
                    act_sent = true;
                }
                const int s = it % S;
                if (it >= S && !mbar_wait(empty0 + 8 * s, ((it / S) & 1) ^ 1)) {
                    ok = false;
                    break;
                }
                const int r0 = (int(blockIdx.x) + int(gridDim.x) * i) * kMmaRows, nr = min(kMmaRows, P.n_out - r0);
                mbar_arrive_tx(full0 + 8 * s, uint32_t(nr * kQ6ChunkBytes));
                for (int r = 0; r < nr; ++r)
                    bulk_g2s(stage0 + uint32_t(s) * slot_bytes + uint32_t(r * kQ6ChunkBytes),
                             P.w + (long long)(r0 + r) * P.row_bytes + (long long)kc * kQ6ChunkBytes, kQ6ChunkBytes,
                             full0 + 8 * s);
            }
            if (!act_sent && ok) {
                if (kc == 0) asm volatile("griddepcontrol.wait;" ::: "memory");
                copy_act();
            }
        }
        if (!ok) {
            if (P.status) atomicOr(P.status, DEV_TIMEOUT);
            for (int k = (it > S ? it - S : 0); k < it; ++k) mbar_wait(full0 + 8 * (k % S), (k / S) & 1);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int cl = threadIdx.x, nthr = 32 * NCW;
    for (int i = cl; i < my_rb * kMmaRows * kMmaMaxTok; i += nthr) run[i] = 0.f;
    const int gid = lane >> 2, tig = lane & 3;
    const int sbw = warp >> 1, nw = warp & 1;           // this warp: superblock sbw of the chunk, half nw
    const bool tok_ok = gid < P.n_tok;                  // B fragment: token gid (zero beyond n_tok)
    const int t0 = 2 * tig, t1 = 2 * tig + 1;           // tokens of this thread's C values
    // up to kQ6RegBlocks row blocks a CTA: each warp keeps its running sums in registers across the
    // chunks and the warps' sums are added once at the end (no barrier per tile); more: per tile
    // through shared memory into `run`
    const bool in_regs = my_rb <= kQ6RegBlocks;
    float racc[kQ6RegBlocks][4];
#pragma unroll
    for (int b = 0; b < kQ6RegBlocks; ++b) racc[b][0] = racc[b][1] = racc[b][2] = racc[b][3] = 0.f;
    float* rw = red + warp * kMmaRows * kMmaMaxTok;
    bool dead = false;
    int it = 0;
    for (int kc = 0; kc < n_kc; ++kc) {
        const int ab = kc & 1;
        const bool agot = !dead && mbar_wait(afull0 + 8 * ab, (kc / 2) & 1);
        if (!agot && !dead) {
            dead = true;
            if (lane == 0 && P.status) atomicOr(P.status, DEV_TIMEOUT);
        }
        const int8_t* axq = reinterpret_cast<const int8_t*>(actb + ab * kQ6ActBytes);
        const int8_t* axq2 = axq + kMmaMaxTok * kQ6ActStride;
        const float* axd = reinterpret_cast<const float*>(axq + 2 * kMmaMaxTok * kQ6ActStride);
        for (int i = 0; i < my_rb; ++i, ++it) {
            const int s = it % S;
            const bool got = !dead && mbar_wait(full0 + 8 * s, (it / S) & 1);
            if (!got && !dead) {
                dead = true;
                if (lane == 0 && P.status) atomicOr(P.status, DEV_TIMEOUT);
            }
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            if (got && sbw < kQ6Chunk / 256) {
                const uint32_t tile = stage0 + uint32_t(s) * slot_bytes;
                const uint32_t bg = tile + uint32_t(gid * kQ6ChunkBytes + sbw * 210);
                const uint32_t bh = tile + uint32_t((gid + 8) * kQ6ChunkBytes + sbw * 210);
                const float dg = h2f(lds16u(bg + 208)), dh = h2f(lds16u(bh + 208));
                const int vbase = sbw * 256 + 128 * nw;      // value index of this half within the chunk
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    // positions 16h + 4 tig.. of half nw: ql runs (groups 0/2 and 1/3) and the qh run
                    const uint32_t lo = 64 * nw + 16 * h + 4 * tig, qo = 128 + 32 * nw + 16 * h + 4 * tig;
                    const uint32_t Lg0 = lds32_a2(bg + lo), Lg1 = lds32_a2(bg + lo + 32), Hg = lds32_a2(bg + qo);
                    const uint32_t Lh0 = lds32_a2(bh + lo), Lh1 = lds32_a2(bh + lo + 32), Hh = lds32_a2(bh + qo);
#pragma unroll
                    for (int grp = 0; grp < 4; ++grp) {
                        const uint32_t Lg = (grp & 1) ? Lg1 : Lg0, Lh = (grp & 1) ? Lh1 : Lh0;
                        const int ls = 4 * (grp >> 1), hs = 2 * grp;
                        const uint32_t a0 = q6_signed(((Lg >> ls) & 0x0F0F0F0Fu) | (((Hg >> hs) & 0x03030303u) << 4));
                        const uint32_t a1 = q6_signed(((Lh >> ls) & 0x0F0F0F0Fu) | (((Hh >> hs) & 0x03030303u) << 4));
                        const int k0 = vbase + 32 * grp + 16 * h + 4 * tig;        // B: token gid, k0..k0+3
                        const uint32_t b = tok_ok ? *reinterpret_cast<const uint32_t*>(axq + gid * kQ6ActStride + k0) : 0u;
                        const uint32_t c = tok_ok ? *reinterpret_cast<const uint32_t*>(axq2 + gid * kQ6ActStride + k0) : 0u;
                        int s1[4] = {0, 0, 0, 0}, s2[4] = {0, 0, 0, 0};
                        mma_s8s8_k16(s1, a0, a1, b);
                        mma_s8s8_k16(s2, a0, a1, c);
                        // scale of this 16-value group (scale index 8 nw + 2 grp + h) and the tokens' xd
                        const int si = 192 + 8 * nw + 2 * grp + h;
                        const float wg = dg * float(int8_t(lds8u(bg + si))), wh = dh * float(int8_t(lds8u(bh + si)));
                        const int blk = (vbase + 32 * grp) / 32;
                        const float x0 = t0 < P.n_tok ? axd[t0 * (kQ6Chunk / 32 + 4) + blk] * kInv254 : 0.f;
                        const float x1 = t1 < P.n_tok ? axd[t1 * (kQ6Chunk / 32 + 4) + blk] * kInv254 : 0.f;
                        acc[0] += wg * x0 * float(254 * s1[0] + s2[0]);
                        acc[1] += wg * x1 * float(254 * s1[1] + s2[1]);
                        acc[2] += wh * x0 * float(254 * s1[2] + s2[2]);
                        acc[3] += wh * x1 * float(254 * s1[3] + s2[3]);
                    }
                }
            }
            __syncwarp();
            if (got && lane == 0) mbar_arrive(empty0 + 8 * s);
            if (in_regs) {
#pragma unroll
                for (int b = 0; b < kQ6RegBlocks; ++b)
                    if (b == i) {
                        racc[b][0] += acc[0];
                        racc[b][1] += acc[1];
                        racc[b][2] += acc[2];
                        racc[b][3] += acc[3];
                    }
                continue;
            }
            rw[gid * kMmaMaxTok + t0] = acc[0];
            rw[gid * kMmaMaxTok + t1] = acc[1];
            rw[(gid + 8) * kMmaMaxTok + t0] = acc[2];
            rw[(gid + 8) * kMmaMaxTok + t1] = acc[3];
            named_sync(kConsumerBarrier, nthr);
            if (cl < kMmaRows * kMmaMaxTok) {
                float v = 0.f;
                for (int w = 0; w < NCW; ++w) v += red[w * kMmaRows * kMmaMaxTok + cl];   // fixed order
                run[i * kMmaRows * kMmaMaxTok + cl] += v;
            }
            named_sync(kConsumerBarrier, nthr);
        }
        if (agot && lane == 0) mbar_arrive(aempty0 + 8 * ab);     // this warp is done with the chunk
    }
    for (int i = 0; i < my_rb; ++i) {
        const int r0 = (int(blockIdx.x) + int(gridDim.x) * i) * kMmaRows;
        if (in_regs) {                                  // the warps' register sums, added in warp order
            float v4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int b = 0; b < kQ6RegBlocks; ++b)
                if (b == i) {
                    v4[0] = racc[b][0];
                    v4[1] = racc[b][1];
                    v4[2] = racc[b][2];
                    v4[3] = racc[b][3];
                }
            rw[gid * kMmaMaxTok + t0] = v4[0];
            rw[gid * kMmaMaxTok + t1] = v4[1];
            rw[(gid + 8) * kMmaMaxTok + t0] = v4[2];
            rw[(gid + 8) * kMmaMaxTok + t1] = v4[3];
            named_sync(kConsumerBarrier, nthr);
            if (cl < kMmaRows * kMmaMaxTok && !dead) {
                const int r = cl / kMmaMaxTok, tk = cl % kMmaMaxTok;
                float v = 0.f;
                for (int w = 0; w < NCW; ++w) v += red[w * kMmaRows * kMmaMaxTok + cl];   // fixed order
                if (tk < P.n_tok && r0 + r < P.n_out) P.y[(long long)tk * P.n_out + r0 + r] = v;
            }
            named_sync(kConsumerBarrier, nthr);
            continue;
        }
        if (cl < kMmaRows * kMmaMaxTok && !dead) {
            const int r = cl / kMmaMaxTok, tk = cl % kMmaMaxTok;
            if (tk < P.n_tok && r0 + r < P.n_out) P.y[(long long)tk * P.n_out + r0 + r] = run[i * kMmaRows * kMmaMaxTok + cl];
        }
    }
}

}  // namespace qmv
