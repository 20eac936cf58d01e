// C ABI of the quantized matvec path (declarations and contracts: include/nemicli_qmv.h).
#include <cstdio>
#include <mutex>

#include "qmv_kernels.cuh"
#include "../../include/nemicli_qmv.h"

using namespace qmv;

namespace {

thread_local int g_last_cuda_error = 0;
__device__ int g_device_status = 0;

int sm_count() {
    static std::mutex mu;
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

int launched() {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        g_last_cuda_error = int(e);
        return ST_LAUNCH;
    }
    return ST_OK;
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

int* device_status_ptr() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
    return static_cast<int*>(p);
}

// common shape/pointer checks of a matvec call
int check_mv(int fmt, const void* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2, const float* xd,
             const float* xs, const void* y) {
    if (!known_format(fmt)) return ST_BAD_FORMAT;
    if (!w || !xq || !xq2 || !xd || !xs || !y) return ST_NULL;
    if (n_out <= 0 || n_in <= 0 || n_in % block_values(fmt)) return ST_BAD_SHAPE;
    if (!aligned(xq, 16) || !aligned(xq2, 16) || !aligned(xd, 8) || !aligned(xs, 8) || !aligned(y, 4))
        return ST_BAD_ALIGN;
    return ST_OK;
}

template <int FMT, int T, bool SUMS>
int launch_t(const MvParams& P, cudaStream_t st) {
    constexpr int RW = 2;
    constexpr int R = SUMS ? 1 : RW;
    const long long groups = (long long)((P.n_out + R - 1) / R) * P.slots;
    long long blocks = (groups + kWarpsPerBlock - 1) / kWarpsPerBlock;
    const long long cap = (long long)sm_count() * 16;
    if (blocks > cap) blocks = cap;
    mv_kernel<FMT, T, R, SUMS><<<unsigned(blocks), 32 * kWarpsPerBlock, 0, st>>>(P);
    return launched();
}

template <int FMT>
int launch_fmt(const MvParams& P, int T, cudaStream_t st) {
    switch (T) {
    case 1: return launch_t<FMT, 1, false>(P, st);
    case 2: return launch_t<FMT, 2, false>(P, st);
    case 3: return launch_t<FMT, 3, false>(P, st);
    case 4: return launch_t<FMT, 4, false>(P, st);
    case 5: return launch_t<FMT, 5, false>(P, st);
    case 6: return launch_t<FMT, 6, false>(P, st);
    case 7: return launch_t<FMT, 7, false>(P, st);
    case 8: return launch_t<FMT, 8, false>(P, st);
    }
    return ST_BAD_TOKENS;
}

int launch(int fmt, const MvParams& P, int T, cudaStream_t st) {
    switch (fmt) {
    case F_Q4_0: return launch_fmt<F_Q4_0>(P, T, st);
    case F_Q8_0: return launch_fmt<F_Q8_0>(P, T, st);
    case F_Q4_K: return launch_fmt<F_Q4_K>(P, T, st);
    case F_Q6_K: return launch_fmt<F_Q6_K>(P, T, st);
    case F_IQ2_XXS: return launch_fmt<F_IQ2_XXS>(P, T, st);
    case F_TQ2_0: return launch_fmt<F_TQ2_0>(P, T, st);
    }
    return ST_BAD_FORMAT;
}

int launch_sums(int fmt, const MvParams& P, cudaStream_t st) {
    switch (fmt) {
    case F_Q4_0: return launch_t<F_Q4_0, 1, true>(P, st);
    case F_Q8_0: return launch_t<F_Q8_0, 1, true>(P, st);
    case F_Q4_K: return launch_t<F_Q4_K, 1, true>(P, st);
    case F_Q6_K: return launch_t<F_Q6_K, 1, true>(P, st);
    case F_IQ2_XXS: return launch_t<F_IQ2_XXS, 1, true>(P, st);
    case F_TQ2_0: return launch_t<F_TQ2_0, 1, true>(P, st);
    }
    return ST_BAD_FORMAT;
}

}  // namespace

extern "C" {

int qmv_abi_version(void) { return NEMICLI_QMV_ABI_VERSION; }

const char* qmv_status_string(int status) {
    switch (status) {
    case ST_OK: return "ok";
    case ST_BAD_FORMAT: return "unsupported block format";
    case ST_BAD_SHAPE: return "bad shape (n_in must be a positive multiple of the block size, n_out > 0)";
    case ST_BAD_ALIGN: return "misaligned pointer";
    case ST_BAD_TOKENS: return "token count out of range";
    case ST_LAUNCH: return "CUDA launch failed";
    case ST_NULL: return "null pointer";
    case ST_DEVICE: return "device status query failed";
    }
    return "unknown status";
}

int qmv_last_cuda_error(void) { return g_last_cuda_error; }

int qmv_block_values(int ggml_type) { return known_format(ggml_type) ? block_values(ggml_type) : 0; }
int qmv_block_bytes(int ggml_type) { return known_format(ggml_type) ? block_bytes(ggml_type) : 0; }

int qmv_supported(int ggml_type, int n_in) {
    return known_format(ggml_type) && n_in > 0 && n_in % block_values(ggml_type) == 0;
}

int qmv_quant_q8(const void* x, int x_is_f32, int8_t* xq, int8_t* xq2, float* xd, float* xs, long long n,
                 void* stream) {
    if (!x || !xq || !xq2 || !xd || !xs) return ST_NULL;
    if (n <= 0 || n % 32) return ST_BAD_SHAPE;
    if (!aligned(x, x_is_f32 ? 4 : 2)) return ST_BAD_ALIGN;
    const long long blocks = (n + 255) / 256;
    quant_q8_kernel<<<unsigned(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(x, x_is_f32, xq, xq2, xd, xs, n);
    return launched();
}

int qmv_mv(int ggml_type, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
           const float* xd, const float* xs, int n_tok, float* y, void* stream) {
    int st = check_mv(ggml_type, w, n_out, n_in, xq, xq2, xd, xs, y);
    if (st) return st;
    if (n_tok <= 0) return ST_BAD_TOKENS;
    if (!aligned(w, ggml_type == F_Q4_K ? 16 : 2)) return ST_BAD_ALIGN;
    MvParams P{};
    P.w = w;
    P.ids = nullptr;
    P.per_expert = 0;
    P.row_bytes = (long long)(n_in / block_values(ggml_type)) * block_bytes(ggml_type);
    P.x_group = 1;
    P.status = device_status_ptr();
    P.n_out = n_out;
    P.n_in = n_in;
    P.slots = 1;
    for (int c0 = 0; c0 < n_tok; c0 += kMaxTokens) {
        const int T = n_tok - c0 < kMaxTokens ? n_tok - c0 : kMaxTokens;
        const long long off = (long long)c0 * n_in;
        P.xq = xq + off;
        P.xq2 = xq2 + off;
        P.xd = xd + off / 32;
        P.xs = xs + off / 32;
        P.y = y + (long long)c0 * n_out;
        if ((st = launch(ggml_type, P, T, static_cast<cudaStream_t>(stream)))) return st;
    }
    return ST_OK;
}

int qmv_mv_experts(int ggml_type, const void* raw, long long per_expert, long long n_exp, const long long* ids, int k,
                   const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int x_group,
                   float* y, int n_out, int n_in, void* stream) {
    int st = check_mv(ggml_type, raw, n_out, n_in, xq, xq2, xd, xs, y);
    if (st) return st;
    if (!ids) return ST_NULL;
    if (k <= 0) return ST_BAD_TOKENS;
    if (n_exp <= 0) return ST_BAD_SHAPE;
    if (x_group <= 0) return ST_BAD_SHAPE;
    const long long row_bytes = (long long)(n_in / block_values(ggml_type)) * block_bytes(ggml_type);
    if (per_expert >= 0) {
        if (per_expert < row_bytes * n_out) return ST_BAD_SHAPE;
        if (!aligned(raw, ggml_type == F_Q4_K ? 16 : 2) || per_expert % (ggml_type == F_Q4_K ? 16 : 2))
            return ST_BAD_ALIGN;
    } else if (!aligned(raw, 8)) {
        return ST_BAD_ALIGN;
    }
    MvParams P{};
    P.w = static_cast<const uint8_t*>(raw);
    P.ids = ids;
    P.per_expert = per_expert >= 0 ? per_expert : -1;
    P.row_bytes = row_bytes;
    P.xq = xq;
    P.xq2 = xq2;
    P.xd = xd;
    P.xs = xs;
    P.x_group = x_group;
    P.y = y;
    P.status = device_status_ptr();
    P.n_out = n_out;
    P.n_in = n_in;
    P.slots = k;
    P.n_exp = n_exp;
    return launch(ggml_type, P, 1, static_cast<cudaStream_t>(stream));
}

int qmv_block_sums(int ggml_type, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
                   int32_t* s, int32_t* s2, void* stream) {
    if (!known_format(ggml_type)) return ST_BAD_FORMAT;
    if (!w || !xq || !xq2 || !s || !s2) return ST_NULL;
    if (n_out <= 0 || n_in <= 0 || n_in % block_values(ggml_type)) return ST_BAD_SHAPE;
    if (!aligned(xq, 16) || !aligned(xq2, 16) || !aligned(s, 4) || !aligned(s2, 4)) return ST_BAD_ALIGN;
    if (!aligned(w, ggml_type == F_Q4_K ? 16 : 2)) return ST_BAD_ALIGN;
    const long long units = (long long)n_out * (n_in / unit_values(ggml_type));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemsetAsync(s, 0, units * sizeof(int32_t), st) != cudaSuccess ||
        cudaMemsetAsync(s2, 0, units * sizeof(int32_t), st) != cudaSuccess) {
        g_last_cuda_error = int(cudaGetLastError());
        return ST_LAUNCH;
    }
    MvParams P{};
    P.w = w;
    P.row_bytes = (long long)(n_in / block_values(ggml_type)) * block_bytes(ggml_type);
    P.xq = xq;
    P.xq2 = xq2;
    P.s = s;
    P.s2 = s2;
    P.status = device_status_ptr();
    P.n_out = n_out;
    P.n_in = n_in;
    P.slots = 1;
    return launch_sums(ggml_type, P, st);
}

int qmv_device_status(int clear, int* out, void* stream) {
    if (!out) return ST_NULL;
    int* p = device_status_ptr();
    if (!p) return ST_DEVICE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(out, p, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return ST_DEVICE;
    if (cudaStreamSynchronize(st) != cudaSuccess) return ST_DEVICE;
    if (clear && cudaMemsetAsync(p, 0, sizeof(int), st) != cudaSuccess) return ST_DEVICE;
    return ST_OK;
}

}  // extern "C"
