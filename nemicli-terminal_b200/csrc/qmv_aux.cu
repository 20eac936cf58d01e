// The small kernels around the matvecs: the fused producers of the activation input for one token
// (RMS norm, gated activation) and the unpacking of block-format matrices to dense values.  C-ABI
// declarations: include/nemicli_qmv.h.
#include <type_traits>

#include "qmv_host.cuh"
#include "qmv_unpack.cuh"
#include "../../include/nemicli_qmv.h"

using namespace qmv;

namespace {

constexpr int kNormThreads = 1024;       // threads of the sum's order (see norm_q8_kernel)
constexpr int kNormBlock = 256;          // threads of a CTA

// RMS norm of one row (ggufengine/mmvq.py:100-118): v = h (+ rs r, written to hout),
// xn = v * rsqrt(mean(v^2) + eps) * w, quantised per 32 values into the activation input.  The sum of
// v^2 has one fixed order, that of 1024 threads where thread t adds v[t], v[t + 1024], ... with fmaf,
// then a warp sum per 32 of them and a warp sum of the 32 results (the order the fused form in the
// staged matvec follows too).  Every CTA forms that sum over the whole row (the row is a few KB, read
// from L2) and then normalises and quantises its own 256 values, one group per warp: no single CTA
// walks the row alone.
__global__ void __launch_bounds__(kNormBlock) norm_q8_kernel(const float* __restrict__ h, const float* __restrict__ r,
                                                             float rs, float* __restrict__ hout,
                                                             const float* __restrict__ w, float eps,
                                                             float* __restrict__ xn, int8_t* __restrict__ xq,
                                                             int8_t* __restrict__ xq2, float* __restrict__ xd,
                                                             float* __restrict__ xs, int n) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");   // the next matvec may stream weights
    asm volatile("griddepcontrol.wait;" ::: "memory");                // inputs and outputs after the previous kernel
    __shared__ float red[32];
    constexpr int K = kNormThreads / kNormBlock;       // order threads per thread: t = p + kNormBlock k
    const int p = threadIdx.x, warp = p >> 5, lane = p & 31;
    const int i = blockIdx.x * kNormBlock + p;         // this thread's own value (second pass)
    const bool own = i - lane < n;                     // the whole warp (n % 32 == 0)
    // loaded together with the first pass's terms: no second round trip to memory after the barrier
    const float hi = own ? h[i] : 0.f, ri = own && r ? r[i] : 0.f, wi = own ? w[i] : 0.f;
    float ss[K];
#pragma unroll
    for (int k = 0; k < K; ++k) ss[k] = 0.f;
    for (int i0 = 0; i0 < n; i0 += 4 * kNormThreads) {             // four of each thread's terms in flight
        float v[4][K];
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int i = i0 + kNormThreads * q + p + kNormBlock * k;
                v[q][k] = i < n ? (r ? __fadd_rn(h[i], __fmul_rn(rs, r[i])) : h[i]) : 0.f;
            }
#pragma unroll
        for (int q = 0; q < 4; ++q)
#pragma unroll
            for (int k = 0; k < K; ++k)
                if (i0 + kNormThreads * q + p + kNormBlock * k < n) ss[k] = __fmaf_rn(v[q][k], v[q][k], ss[k]);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {                      // order warp (p + kNormBlock k) / 32 = warp + 8 k
        const float t = warp_sum(ss[k]);
        if (lane == 0) red[warp + (kNormBlock / 32) * k] = t;
    }
    __syncthreads();
    const float inv = rsqrtf(warp_sum(red[lane]) / float(n) + eps);
    if (own) {
        const float v = r ? __fadd_rn(hi, __fmul_rn(rs, ri)) : hi;
        if (r) hout[i] = v;
        const float x = __fmul_rn(__fmul_rn(v, inv), wi);
        xn[i] = x;
        quantize_group(x, i, xq, xq2, xd, xs);
    }
}

// a = act(g) * u (u null: act(g)), act = SiLU or GELU (tanh form) (ggufengine/mmvq.py:120-131), and its
// activation input; one warp per 32 values.
__global__ void __launch_bounds__(256) act_q8_kernel(const float* __restrict__ g, const float* __restrict__ u, int gelu,
                                                     float* __restrict__ a, int8_t* __restrict__ xq,
                                                     int8_t* __restrict__ xq2, float* __restrict__ xd,
                                                     float* __restrict__ xs, int n) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if ((i & ~31) >= n) return;                       // whole warps: n % 32 == 0
    const float v = act_value(g[i], u ? u[i] : 0.f, u != nullptr, gelu);
    a[i] = v;
    quantize_group(v, i, xq, xq2, xd, xs);
}

template <class Fn>
int by_format(int fmt, Fn&& f) {
#define QMV_CASE(F) case F: return f(std::integral_constant<int, F>{});
    switch (fmt) {
    QMV_CASE(F_Q4_0) QMV_CASE(F_Q4_1) QMV_CASE(F_Q5_0) QMV_CASE(F_Q5_1) QMV_CASE(F_Q8_0) QMV_CASE(F_IQ4_NL)
    QMV_CASE(F_MXFP4) QMV_CASE(F_Q1_0) QMV_CASE(F_Q2_0) QMV_CASE(F_PQ2_0) QMV_CASE(F_Q2_K) QMV_CASE(F_Q3_K)
    QMV_CASE(F_Q4_K) QMV_CASE(F_Q5_K) QMV_CASE(F_Q6_K) QMV_CASE(F_IQ2_XXS) QMV_CASE(F_IQ2_XS) QMV_CASE(F_IQ2_S)
    QMV_CASE(F_IQ3_XXS) QMV_CASE(F_IQ3_S) QMV_CASE(F_IQ4_XS) QMV_CASE(F_TQ1_0) QMV_CASE(F_TQ2_0)
    QMV_CASE(F_IQ1_S) QMV_CASE(F_IQ1_M) QMV_CASE(F_PTQ1_0)
    }
#undef QMV_CASE
    return ST_BAD_FORMAT;
}

template <int FMT>
int launch_unpack(const uint8_t* w, long long n_values, void* out, int out_dtype, cudaStream_t st) {
    const long long threads = n_values / 8;
    const long long blocks = (threads + 255) / 256;
    if (blocks > 0x7FFFFFFFLL) return ST_BAD_SHAPE;
    switch (out_dtype) {
    case QMV_OUT_F32: unpack_kernel<FMT, 0><<<unsigned(blocks), 256, 0, st>>>(w, out, n_values); break;
    case QMV_OUT_BF16: unpack_kernel<FMT, 1><<<unsigned(blocks), 256, 0, st>>>(w, out, n_values); break;
    case QMV_OUT_F16: unpack_kernel<FMT, 2><<<unsigned(blocks), 256, 0, st>>>(w, out, n_values); break;
    default: return ST_BAD_SHAPE;
    }
    return launched();
}

}  // namespace

extern "C" {

int qmv_norm_q8(const float* h, const float* r, float rs, float* h_out, const float* w, float eps, float* xn,
                int8_t* xq, int8_t* xq2, float* xd, float* xs, int n, void* stream) {
    if (!h || !w || !xn || !xq || !xq2 || !xd || !xs || (r && !h_out)) return ST_NULL;
    if (n <= 0 || n % 32) return ST_BAD_SHAPE;
    if (!aligned(xq, 16) || !aligned(xq2, 16) || !aligned(xd, 4) || !aligned(xs, 4)) return ST_BAD_ALIGN;
    return launch_pdl(norm_q8_kernel, dim3((n + kNormBlock - 1) / kNormBlock), dim3(kNormBlock),
                      static_cast<cudaStream_t>(stream), h, r, rs, h_out, w, eps, xn, xq, xq2, xd, xs, n);
}

int qmv_act_q8(const float* g, const float* u, int gelu, float* a, int8_t* xq, int8_t* xq2, float* xd, float* xs,
               int n, void* stream) {
    if (!g || !a || !xq || !xq2 || !xd || !xs) return ST_NULL;
    if (n <= 0 || n % 32) return ST_BAD_SHAPE;
    if (!aligned(xq, 16) || !aligned(xq2, 16) || !aligned(xd, 4) || !aligned(xs, 4)) return ST_BAD_ALIGN;
    return launch_pdl(act_q8_kernel, dim3((n + 255) / 256), dim3(256), static_cast<cudaStream_t>(stream), g, u, gelu,
                      a, xq, xq2, xd, xs, n);
}

int qmv_unpack(int ggml_type, const uint8_t* w, long long n_values, void* out, int out_dtype, void* stream) {
    if (!known_format(ggml_type)) return ST_BAD_FORMAT;
    if (!w || !out) return ST_NULL;
    if (n_values <= 0 || n_values % block_values(ggml_type)) return ST_BAD_SHAPE;
    if (!aligned(out, 16)) return ST_BAD_ALIGN;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    return by_format(ggml_type, [&](auto c) {
        return launch_unpack<decltype(c)::value>(w, n_values, out, out_dtype, st);
    });
}

}  // extern "C"
