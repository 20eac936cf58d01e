// Few-token (2..8 tokens) matvec on the tensor cores: host side of the kernels in qmv_mma.cuh.
#include <algorithm>

#include "qmv_host.cuh"
#include "qmv_mma.cuh"

namespace qmv {
namespace {

// Few-token Q4_K / Q8_0 matvec on the tensor cores, 1..kMmaJobs matrices of the same row length reading
// the same tokens in one launch; false when the shape or alignment does not qualify.
template <int FMT>
bool mma_dense_k(int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                 long long row_bytes, const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int T,
                 cudaStream_t st, int* status) {
    if (T < 2 || T > kMmaMaxTok || n_in % block_values(FMT) || n_in > kMmaMaxIn || !tma_enabled()) return false;
    if (n_jobs < 1 || n_jobs > kMmaJobs || !aligned(xq, 16) || !aligned(xq2, 16) || row_bytes % 16) return false;
    for (int j = 0; j < n_jobs; ++j)
        if (!aligned(w[j], 16) || n_out[j] <= 0) return false;
    constexpr int NCW = 16;
    const long long other = mma_act_bytes(n_in) + mma_red_bytes(NCW) + 2 * 8 * 32;
    const long long slot = kMmaRows * mma_row_stride(row_bytes);
    long long S = (kSmemCap - other) / slot;
    if (S > 4) S = 4;
    if (S < 2) return false;
    MmaParams P{};
    P.w = w[0]; P.y = y[0]; P.xq = xq; P.xq2 = xq2; P.xd = xd; P.xs = xs;
    P.row_bytes = row_bytes; P.n_out = n_out[0]; P.n_in = n_in; P.n_tok = T; P.stages = int(S);
    P.status = device_status_ptr();
    P.n_jobs = n_jobs;
    int tiles = 0;
    for (int j = 0; j < n_jobs; ++j) {
        P.jw[j] = w[j];
        P.jy[j] = y[j];
        P.jn[j] = n_out[j];
        P.jt[j] = tiles;
        tiles += (n_out[j] + kMmaRows - 1) / kMmaRows;
    }
    P.jt[n_jobs] = tiles;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(mv_mma_kernel<FMT, NCW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess) {
            *status = launched();
            return true;
        }
        configured[dev] = 1;
    }
    const int grid = std::min(tiles, sm_count());
    *status = launch_pdl_smem(mv_mma_kernel<FMT, NCW>, dim3(grid), dim3(32 * (NCW + 1)), size_t(S * slot + other), st, P);
    return true;
}
}  // namespace

bool mma_q4k(const uint8_t* w, int n_out, int n_in, long long row_bytes, const int8_t* xq, const int8_t* xq2,
             const float* xd, const float* xs, int T, float* y, int fmt, cudaStream_t st, int* status) {
    return mma_q4k_multi(1, &w, &n_out, &y, n_in, row_bytes, xq, xq2, xd, xs, T, fmt, st, status);
}

bool mma_q4k_multi(int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                   long long row_bytes, const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int T,
                   int fmt, cudaStream_t st, int* status) {
    if (fmt == F_Q4_K)
        return mma_dense_k<F_Q4_K>(n_jobs, w, n_out, y, n_in, row_bytes, xq, xq2, xd, xs, T, st, status);
    if (fmt == F_Q8_0)
        return mma_dense_k<F_Q8_0>(n_jobs, w, n_out, y, n_in, row_bytes, xq, xq2, xd, xs, T, st, status);
    return false;
}

// Few-token Q6_K matvec on the tensor cores (rows of a multiple of 2048 values).
bool mma_q6k(const uint8_t* w, int n_out, int n_in, long long row_bytes, const int8_t* xq, const int8_t* xq2,
             const float* xd, int T, float* y, int fmt, cudaStream_t st, int* status) {
    if (fmt != F_Q6_K || T < 2 || T > kMmaMaxTok || n_in % kQ6Chunk || !tma_enabled()) return false;
    if (!aligned(w, 16) || !aligned(xq, 16) || !aligned(xq2, 16) || row_bytes % 16) return false;
    constexpr int NCW = 16;
    const int n_rb = (n_out + kMmaRows - 1) / kMmaRows;
    const int grid = std::min(n_rb, sm_count());
    if ((n_rb + grid - 1) / grid > kQ6MaxBlocks) return false;
    if (!aligned(xd, 16)) return false;
    const long long other = 2LL * kQ6ActBytes + mma_red_bytes(NCW) + 4LL * kQ6MaxBlocks * kMmaRows * kMmaMaxTok + 2 * 8 * 32;
    const long long slot = (long long)kMmaRows * kQ6ChunkBytes;
    long long S = (kSmemCap - other) / slot;
    if (S > 6) S = 6;
    if (S < 2) return false;
    MmaParams P{};
    P.w = w; P.y = y; P.xq = xq; P.xq2 = xq2; P.xd = xd; P.xs = nullptr;
    P.row_bytes = row_bytes; P.n_out = n_out; P.n_in = n_in; P.n_tok = T; P.stages = int(S);
    P.status = device_status_ptr();
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(mv_mma_q6k_kernel<NCW>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap) != cudaSuccess) {
            *status = launched();
            return true;
        }
        configured[dev] = 1;
    }
    *status = launch_pdl_smem(mv_mma_q6k_kernel<NCW>, dim3(grid), dim3(32 * (NCW + 1)), size_t(S * slot + other), st,
                              P);
    return true;
}
}  // namespace qmv
