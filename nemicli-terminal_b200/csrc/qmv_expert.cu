// Expert-parallel MoE exchange on the device (shard.ExpertShardedMoE): the send buffer of a call built in
// two launches instead of a chain of tensor operations, and the home rank's weighted slot sum in one.
// C-ABI declarations: include/nemicli_qmv.h.
//
// Send buffer: world blocks of P = n_tok * k slots, a slot = one row of row_floats floats (the pair's
// activation in [0, dim), then its owner-local expert id as an exact float, then padding).  Pair p goes
// to the owner of its expert (experts split by whole items as shard_range does, the first n_exp % world
// ranks one more) at the next free position of that owner's block (pairs in index order); an id outside
// [0, n_exp) goes to rank 0 with id -2 (the owner's kernels give zeros and the device status bit); every
// slot no pair takes gets id -1 (its row is not written: the kernels never read an unused slot's data).
#include <algorithm>

#include "qmv_host.cuh"
#include "../../include/nemicli_qmv.h"

using namespace qmv;

namespace {

constexpr int kDispatchThreads = 1024;
constexpr int kMaxWorld = 64;

__device__ __forceinline__ int owner_of(long long e, long long n_exp, int world, long long* lo) {
    const long long base = n_exp / world, extra = n_exp % world, big = extra * (base + 1);
    const int r = e < big ? int(e / (base + 1)) : int(extra + (e - big) / (base > 0 ? base : 1));
    *lo = (long long)r * base + (r < extra ? r : extra);
    return r;
}

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// one CTA: slot of every pair, the id column of every slot, the pairs sent to each rank
__global__ void __launch_bounds__(kDispatchThreads) dispatch_index_kernel(const long long* __restrict__ ids, int P,
                                                                          long long n_exp, int world,
                                                                          float* __restrict__ send, int row_floats,
                                                                          int dim, long long* __restrict__ slot,
                                                                          int* __restrict__ sent) {
    __shared__ int cur[kMaxWorld];
    for (long long s = threadIdx.x; s < (long long)world * P; s += blockDim.x) send[s * row_floats + dim] = -1.0f;
    if (threadIdx.x < world) cur[threadIdx.x] = 0;
    __syncthreads();
    if (threadIdx.x < 32) {                     // pairs in index order, 32 at a time
        const int lane = threadIdx.x;
        for (int p0 = 0; p0 < P; p0 += 32) {
            const int p = p0 + lane;
            int d = -1;
            float id = 0.f;
            if (p < P) {
                const long long e = ids[p];
                if (e >= 0 && e < n_exp) {
                    long long lo;
                    d = owner_of(e, n_exp, world, &lo);
                    id = float(e - lo);
                } else {
                    d = 0;
                    id = -2.0f;
                }
            }
            const unsigned same = __match_any_sync(0xffffffffu, d);
            int pos = 0;
            if (d >= 0) pos = cur[d] + __popc(same & lanemask_lt());
            __syncwarp();
            if (d >= 0) {
                const long long s = (long long)d * P + pos;
                slot[p] = s;
                send[s * row_floats + dim] = id;
                for (int c = dim + 1; c < row_floats; ++c) send[s * row_floats + c] = 0.f;
                if ((same & lanemask_lt()) == 0) cur[d] += __popc(same);
            }
            __syncwarp();
        }
        __syncwarp();
        if (lane < world) sent[lane] = cur[lane];
    }
}

// CTA p: the activation row of pair p's token into its slot (fp32)
__global__ void __launch_bounds__(256) dispatch_rows_kernel(const void* __restrict__ x, int x_f32, int k, int dim,
                                                            const long long* __restrict__ slot, float* __restrict__ send,
                                                            int row_floats) {
    const int p = blockIdx.x;
    const long long t = p / k;
    float* dst = send + slot[p] * row_floats;
    for (int c = threadIdx.x; c < dim; c += blockDim.x)
        dst[c] = x_f32 ? static_cast<const float*>(x)[t * dim + c] : bf2f(static_cast<const uint16_t*>(x)[t * dim + c]);
}

// out[t][c] = sum_j w[t][j] y[slot[t k + j]][c], slot order, each product then each sum rounded
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ y, int y_stride,
                                                      const long long* __restrict__ slot, const float* __restrict__ w,
                                                      int k, int dim, float* __restrict__ out) {
    const int t = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= dim) return;
    float v = 0.f;
    for (int j = 0; j < k; ++j) {
        const float term = __fmul_rn(y[slot[t * k + j] * y_stride + c], w[t * k + j]);
        v = j == 0 ? term : __fadd_rn(v, term);
    }
    out[(long long)t * dim + c] = v;
}

}  // namespace

extern "C" {

int qmv_expert_dispatch(const long long* ids, int n_tok, int k, long long n_exp, int world, const void* x,
                        int x_is_f32, int dim, float* send, int row_floats, long long* slot, int* sent, void* stream) {
    if (!ids || !x || !send || !slot || !sent) return ST_NULL;
    if (n_tok <= 0 || k <= 0) return ST_BAD_TOKENS;
    if (n_exp <= 0 || world <= 0 || world > kMaxWorld || dim <= 0 || row_floats < dim + 1 ||
        (long long)n_tok * k > (1LL << 24))
        return ST_BAD_SHAPE;
    const int P = n_tok * k;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    dispatch_index_kernel<<<1, kDispatchThreads, 0, st>>>(ids, P, n_exp, world, send, row_floats, dim, slot, sent);
    int rc = launched();
    if (rc) return rc;
    dispatch_rows_kernel<<<P, 256, 0, st>>>(x, x_is_f32, k, dim, slot, send, row_floats);
    return launched();
}

int qmv_expert_combine(const float* y, int y_stride, const long long* slot, const float* w, int n_tok, int k, int dim,
                       float* out, void* stream) {
    if (!y || !slot || !w || !out) return ST_NULL;
    if (n_tok <= 0 || k <= 0) return ST_BAD_TOKENS;
    if (dim <= 0 || y_stride < dim || n_tok > 65535) return ST_BAD_SHAPE;
    const dim3 grid((dim + 255) / 256, n_tok);
    combine_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, y_stride, slot, w, k, dim, out);
    return launched();
}

}  // extern "C"
