// Host-side declarations shared by the library's translation units.
//
// The library is split so that nvcc can build it in parallel: qmv_fmt.cu is compiled once per block
// format (-DQMV_FMT_ID=<GGML type id>) and holds every kernel instantiation of that format; qmv_mma.cu the
// few-token tensor-core kernels; qmv_chain.cu the decode chain; qmv_capi.cu the C ABI that dispatches to
// them.  Kernels receive every device address as a parameter, so no translation unit names another
// one's device symbols.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "qmv_common.cuh"
#include "qmv_kernels.cuh"
#include "qmv_tma.cuh"

namespace qmv {

constexpr int kSmemCap = 232448;          // dynamic shared memory per block on sm_100a (227 KB)
constexpr int kSmemHalf = 113 * 1024;     // two CTAs per SM (the next kernel's CTA can prefetch alongside)

// geometry of one staged (mv_tma_kernel) launch: consumer warps, team width, units per lane, rows per
// tile, ring slots, dynamic shared memory
struct TmaPlan {
    int NCW, G, UPL, R, S, smem;
};

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

// ---- defined in qmv_capi.cu ----
int sm_count();                 // SMs of the current device
int launched();                 // ST_LAUNCH (error recorded for qmv_last_cuda_error) if the last launch failed
void set_last_cuda_error(int e);
int* device_status_ptr();       // the device status word of the current device (null if unavailable)
bool pdl_enabled();             // qmv_set_pdl
bool tma_enabled();             // the staged / tensor-core kernels may be used (sweep builds can turn them off)

// a kernel launch with programmatic dependent launch when qmv_set_pdl is on (the kernel must take
// griddepcontrol.wait before it touches memory); plain stream order otherwise
template <class... KArgs, class... Args>
int launch_pdl_smem(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
    return launched();
}
template <class... KArgs, class... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
    return launch_pdl_smem(kern, grid, block, 0, st, args...);
}

// ---- defined per format in qmv_fmt.cu (one object file per format) ----
// fallback kernel, T = 1..8 tokens
template <int FMT> int launch_mv_fmt(const MvParams& P, int T, cudaStream_t st);
// fallback kernel in int32-sums mode (test hook)
template <int FMT> int launch_sums_fmt(const MvParams& P, cudaStream_t st);
// staged single-token kernel; xf: 0 pre-quantised input, 1 fp32 row, 2 bf16 row quantised in the kernel;
// sums: int32-sums mode (xf == 0 only)
template <int FMT> int launch_tma_fmt(int xf, bool sums, const TmaParams& P, const TmaPlan& pl, int grid,
                                      cudaStream_t st);

struct MoeParams;
// grouped MoE kernels (qmv_moe.cuh): stage 0 gate/up (FMT = gate and up format), 1 down (FMT = down format)
template <int FMT> int launch_moe_fmt(int stage, const MoeParams& P, int grid, cudaStream_t st);

// ---- defined in qmv_mma.cu ----
// few-token (2..8) tensor-core kernels; false when the shape or alignment does not qualify (then the
// caller uses the fallback kernel), true with *status set otherwise
bool mma_q4k(const uint8_t* w, int n_out, int n_in, long long row_bytes, const int8_t* xq, const int8_t* xq2,
             const float* xd, const float* xs, int T, float* y, int fmt, cudaStream_t st, int* status);
// the same for 1..4 matrices of one row length that read the same tokens, in one launch
bool mma_q4k_multi(int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                   long long row_bytes, const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int T,
                   int fmt, cudaStream_t st, int* status);
bool mma_q6k(const uint8_t* w, int n_out, int n_in, long long row_bytes, const int8_t* xq, const int8_t* xq2,
             const float* xd, int T, float* y, int fmt, cudaStream_t st, int* status);

}  // namespace qmv
