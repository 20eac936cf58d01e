/*
 * nemicli_qmv.h — C ABI of the B200 quantized matrix-vector path (GGUF block weights x activations).
 *
 * Plain pointers and sizes only.  Every pointer is a CUDA device pointer (or host memory the GPU
 * can address) unless a comment says otherwise; `stream` is a cudaStream_t (0: the legacy default
 * stream).  Every call only enqueues work on `stream` and returns a status: 0 = ok, else one of
 * QMV_ERR_* (qmv_status_string explains it).  Nothing is allocated and nothing is read back on the
 * host, so the calls can be captured in a CUDA graph.  There is no CPU fallback: a shape, format
 * or alignment the kernels cannot take is refused with a status.
 *
 * Activation input (the reference's "Eingang", ggufengine/mmvq.py:825-849): for n values (n % 32 == 0)
 *   xq  int8[n]    q  = rint(x / d),            d = max|x| / 127 per 32 values
 *   xq2 int8[n]    q2 = rint((x - q d) / (d / 254)) clamped to +-127
 *   xd  float[n/32] d
 *   xs  float[n/32] sum of the 32 values of x
 * Token t of a multi-token input starts at value t * n_in (xq, xq2) and t * n_in / 32 (xd, xs).
 * Alignment: xq, xq2 16 bytes; xd, xs 8 bytes.
 *
 * Weights stay in raw GGUF block layout, row-major (n_out rows of n_in / block_values blocks).
 * Formats (GGML type ids): Q4_0 = 2, Q4_1 = 3, Q5_0 = 6, Q5_1 = 7, Q8_0 = 8, Q2_K = 10, Q3_K = 11, Q4_K = 12, Q5_K = 13, Q6_K = 14, IQ2_XXS = 16, IQ2_XS = 17, IQ3_XXS = 18,
 *          IQ1_S = 19, IQ4_NL = 20, IQ3_S = 21, IQ2_S = 22, IQ4_XS = 23, IQ1_M = 29, TQ1_0 = 34, TQ2_0 = 35, MXFP4 = 39,
 *          Q1_0 = 41, Q2_0 = 42, PQ2_0 = 142 (the reference's id for Q2_0 codes in 128-value blocks), PTQ1_0 = 143
 *          (the reference's id for TQ1_0 trits in 128-value blocks).
 * Alignment: Q4_K and Q5_K weights 16 bytes, MXFP4 4 bytes, the other formats 2 bytes.
 */
#ifndef NEMICLI_QMV_H
#define NEMICLI_QMV_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NEMICLI_QMV_ABI_VERSION 2

#define QMV_OK 0
#define QMV_ERR_FORMAT 1   /* format not one of the twenty-six above */
#define QMV_ERR_SHAPE 2    /* n_in not a positive multiple of the block size, n_out <= 0, ... */
#define QMV_ERR_ALIGN 3    /* a pointer or stride misses the alignment above */
#define QMV_ERR_TOKENS 4   /* token / slot count out of range */
#define QMV_ERR_LAUNCH 5   /* CUDA refused the launch (qmv_last_cuda_error has the cudaError_t) */
#define QMV_ERR_NULL 6     /* a required pointer is null */
#define QMV_ERR_DEVICE 7   /* the device status word could not be read */
#define QMV_ERR_TOO_LARGE 8 /* a size beyond the fixed maximum of a no-allocation entry point */

/* Bits of the device status word (qmv_device_status). */
#define QMV_DEV_BAD_ADDRESS 1   /* an expert id was outside [0, n_exp) or an address-table entry misaligned */

int qmv_abi_version(void);
const char* qmv_status_string(int status);
int qmv_last_cuda_error(void);

/* Values / bytes per block of a format (0 for a format this library does not compute).
 * Replaces: ggufengine/gguf.py:64-77 (GGML_TYPES) for the twenty-six formats. */
int qmv_block_values(int ggml_type);
int qmv_block_bytes(int ggml_type);

/* 1 when the kernels take this format and row length.
 * Replaces: ggufengine/mmvq.py:808 (verfuegbar) and ggufengine/cudakern.py:733 (verfuegbar). */
int qmv_supported(int ggml_type, int n_in);

/* Quantise n values (fp32 if x_is_f32, else bf16) into an activation input.
 * Replaces: ggufengine/mmvq.py:77-83 (quant_q8 kernel) as launched by Eingang.__init__ (:829-843). */
int qmv_quant_q8(const void* x, int x_is_f32, int8_t* xq, int8_t* xq2, float* xd, float* xs, long long n,
                 void* stream);

/* y[t][r] = W[r, :] . x_t for n_tok tokens (any n_tok >= 1; launched in groups of 8), fp32 output
 * [n_tok][n_out].  Replaces: ggufengine/mmvq.py:852-865 (mv: int8 path, Q4_K/Q6_K) and
 * ggufengine/cudakern.py:777-790 (mm) / qlinear.py:210-215 (QuantLinear._mm) for the dense formats. */
int qmv_mv(int ggml_type, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
           const float* xd, const float* xs, int n_tok, float* y, void* stream);

/* Grouped expert matvec driven by device-side ids: y[j][r] = W_{ids[j]}[r, :] . x_{j / x_group}, j < k.
 * raw: the expert tensor (n_exp experts of per_expert bytes each) or, with per_expert < 0, a device
 * table of n_exp int64 addresses (one per expert).  Slot j reads activation row j / x_group (rows are
 * n_in values apart): x_group = k shares one input among all slots, 1 gives each slot its own row,
 * and k_per_token for tokens x slots.  An id of -1 marks an unused slot (a padded exchange buffer):
 * zero rows, no weight read, no error.  Other ids outside [0, n_exp) give zero rows and set
 * QMV_DEV_BAD_ADDRESS.  Replaces: ggufengine/cudakern.py:756-774 (mv, the mv_<FMT> expert gather
 * :483-505) as called by PackedExperts.matvec / matvec_je (models/common.py:462-475). */
int qmv_mv_experts(int ggml_type, const void* raw, long long per_expert, long long n_exp, const long long* ids,
                   int k, const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs,
                   int x_group, float* y, int n_out, int n_in, void* stream);

/* Expert-parallel exchange, send side: pair p = t * k + j of the n_tok x k device ids goes to the rank
 * holding its expert (experts split over `world` ranks by whole items, the first n_exp % world ranks
 * one more) at the next free slot of that rank's block of P = n_tok * k slots (pairs in index order).
 * send: world * P rows of row_floats floats (>= dim + 1): the token's activation (x fp32 if x_is_f32,
 * else bf16) in [0, dim), the owner-local expert id as a float at dim, zeros after; ids outside
 * [0, n_exp) go to rank 0 with id -2, slots no pair takes get id -1 (their data is not written).
 * slot: P int64 (the pair's row in send), sent: world int32 (pairs per rank).  Two launches.
 * Replaces: nothing in the reference (single-GPU); the dispatch of shard.ExpertShardedMoE. */
int qmv_expert_dispatch(const long long* ids, int n_tok, int k, long long n_exp, int world, const void* x,
                        int x_is_f32, int dim, float* send, int row_floats, long long* slot, int* sent, void* stream);

/* Expert-parallel exchange, home side: out[t][c] = sum_j w[t][j] * y[slot[t k + j]][c] over j = 0..k-1
 * in slot order (each product and sum rounded; y rows y_stride floats apart).  One launch.  Replaces:
 * nothing in the reference; the weighted sum of shard.ExpertShardedMoE (the order of moe.py:319-321). */
int qmv_expert_combine(const float* y, int y_stride, const long long* slot, const float* w, int n_tok, int k, int dim,
                       float* out, void* stream);

/* Bytes of the workspace qmv_mm_tc needs (0 for an unsupported format or shape). */
int64_t qmv_mm_tc_workspace_bytes(int ggml_type, int n_out, int n_in, int n_tok);

/* Several tokens on the 5th-generation tensor cores (Q4_K and Q6_K, n_in a multiple of 256): y[t][r] =
 * xs[t] * sum_k fp16(W[r, k]) fp16(x[t, k] / xs[t]) with xs[t] = max|x[t, :]| / 256, fp32 sums, y fp32
 * [n_tok][n_out] overwritten; the weight values are unpacked to fp16 as the reference does (Q4_K d sc q -
 * dmin m in one fused multiply-add, Q6_K d sc (q - 32)).  Tokens go in groups of 128; K is split over
 * the SMs and the parts added in a fixed order (deterministic).  x fp32 if x_is_f32, else bf16;
 * workspace 256-byte aligned, workspace_bytes long: at least qmv_mm_tc_workspace_bytes (else
 * QMV_ERR_SHAPE, nothing launched).  Replaces: ggufengine/mmvq.py:536-724
 * (MMQ: mmq_eingang and mmq_<FMT>_<NT>) as dispatched by mmvq.mm (:902-918) for MMVQ_BIS < M <=
 * MMQ_BIS (models/common.py:406-407). */
int qmv_mm_tc(int ggml_type, const uint8_t* w, int n_out, int n_in, const void* x, int x_is_f32, int n_tok,
              float* y, void* workspace, long long workspace_bytes, void* stream);

/* Bytes of the workspace qmv_moe_ffn needs for n_tok tokens of k slots (0 for an invalid shape). */
int64_t qmv_moe_workspace_bytes(int n_tok, int k, int dim, int ff);

/* Whole mixture-of-experts FFN of n_tok tokens with k slots each (n_tok * k at most 1024, n_exp at most
 * 1024) in three launches:
 *     out[t][:] = sum_j wts[t][j] * down_e(silu(gate_e x_t) * up_e x_t),   e = ids[t][j]
 * x: n_tok rows of dim values, x_stride values apart (fp32 if x_is_f32, else bf16), quantised once;
 * gate and up share one format (n_exp experts of gate_up_per_expert bytes, ff rows of dim values);
 * down has its own (dim rows of ff values).  Every expert the call touches is read once whatever
 * number of tokens chose it; silu and the product are formed and quantised in the gate/up kernel, and
 * the weighted sum over the slots (in slot order) in the down kernel, which writes out (n_tok x dim
 * fp32).  Ids: -1 marks an unused slot (adds nothing); other ids outside [0, n_exp) add nothing and
 * set QMV_DEV_BAD_ADDRESS.  dim and ff multiples of 32 and of their formats' block; workspace 256-byte
 * aligned, qmv_moe_workspace_bytes long.  Replaces: ggufengine/models/moe.py:264-321
 * (Experten.__call__ over PackedExperts with the SiLU gate, models/common.py:462-475) and its
 * cudakern.py:756-774 expert matvecs. */
int qmv_moe_ffn(int gate_up_type, const void* gate, const void* up, long long gate_up_per_expert, int down_type,
                const void* down, long long down_per_expert, long long n_exp, const long long* ids, const float* wts,
                int n_tok, int k, const void* x, int x_is_f32, long long x_stride, int dim, int ff, void* workspace,
                float* out, void* stream);

/* Several matrices reading the same single-token input in one launch (q/k/v, gate/up): for j < n_jobs
 * (at most 4), y[j][r] = W_j[r, :] . x.  w, n_out, y: host arrays of n_jobs entries (device pointers).
 * Replaces: the separate mmvq.mv calls the reference makes for matrices sharing an Eingang
 * (ggufengine/models/baukasten.py:222-240, _mal per matrix). */
int qmv_mv_multi(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                 const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, void* stream);

/* qmv_mv_multi for n_tok tokens (Eingang rows of n_in values; y[j] holds n_tok rows of n_out[j] floats):
 * per group of up to 8 tokens, Q4_K and Q8_0 matrices (rows up to 4096 values) in one tensor-core launch
 * for all n_jobs matrices, other formats one qmv_mv call per matrix.  Replaces: the reference's separate
 * mmvq.mv calls on a shared Eingang for q/k/v and gate/up at 2..16 tokens
 * (ggufengine/models/common.py:404-407, ggufengine/mmvq.py:852-865). */
int qmv_mv_multi_tok(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                     const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int n_tok, void* stream);

/* Single token, raw activation: like qmv_mv_multi, but x (n_in values, fp32 if x_is_f32 else bf16) is
 * quantised inside the kernel (the same arithmetic as qmv_quant_q8), so no activation buffers and no
 * separate launch are needed.  Returns QMV_ERR_SHAPE for a row length the staged kernel does not take
 * (then quantise with qmv_quant_q8 and call qmv_mv).  Replaces: Eingang(x) + mv in one call
 * (ggufengine/mmvq.py:829-865), as PackedLinear._rechnen does for one token (models/common.py:404-405). */
int qmv_mv_x(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
             const void* x, int x_is_f32, void* stream);

/* qmv_mv_multi (one token, pre-quantised input) that also forms the NEXT matvec's activation input from
 * its own outputs: ep_kind 1 quantises y[ep_j0] (as qmv_quant_q8 would, bit for bit); ep_kind 2 forms
 * a = SiLU(y[ep_j0]) * y[ep_j1] into ep_a and quantises it (as qmv_act_q8 with gelu = 0 would).  The CTA
 * that writes the last rows of a 32-row group does that group, so no producer launch follows the
 * matvec.  ep_counters: n_out[ep_j0] / 32 ints, zero before the first call; each call leaves them zero
 * again (calls sharing them must not overlap).  n_out[ep_j0] % 32 == 0 (ep_kind 2: the same n_out for
 * both jobs).  Returns QMV_ERR_SHAPE where the staged kernel cannot do it (then qmv_mv_multi and the
 * producer).  Replaces: mv + Eingang / akt_q8 on its outputs in the reference's one-token step
 * (ggufengine/models/baukasten.py:222-240, ggufengine/mmvq.py:959-966). */
int qmv_mv_multi_ep(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                    const int8_t* xq, const int8_t* xq2, const float* xd, const float* xs, int ep_kind, int ep_j0,
                    int ep_j1, int* ep_counters, int8_t* ep_xq, int8_t* ep_xq2, float* ep_xd, float* ep_xs,
                    float* ep_a, void* stream);

/* Single token, RMS norm fused in front: qmv_norm_q8 (h, r, rs, h_out, norm_w, eps; n = n_in) followed by
 * qmv_mv_multi on its activation input, in one launch.  The quantised input is bit-identical to
 * qmv_norm_q8's (the same order of the sum of squares and the same roundings), so are the outputs; xn is
 * not written.  h_out (given with r) is written once.  Returns QMV_ERR_SHAPE for a row length the staged
 * kernel does not take (then call qmv_norm_q8 and qmv_mv_multi).  Replaces: norm_q8 + the mv calls on
 * its Eingang in the reference's one-token step (ggufengine/models/baukasten.py:205-240,
 * ggufengine/mmvq.py:946-956). */
int qmv_mv_norm(int ggml_type, int n_jobs, const uint8_t* const* w, const int* n_out, float* const* y, int n_in,
                const float* h, const float* r, float rs, float* h_out, const float* norm_w, float eps, void* stream);

/* ---- fused producers of the activation input (one token) and unpacking --------------------------- */

/* RMS norm of one row and its activation input: v = h (+ rs * r, written to h_out when r is given),
 * xn = v * rsqrt(mean(v^2) + eps) * w (n fp32 values, n % 32 == 0), quantised into xq, xq2, xd, xs.
 * One launch.  Replaces: ggufengine/mmvq.py:946-956 (norm_q8) and its kernel (:100-118). */
int qmv_norm_q8(const float* h, const float* r, float rs, float* h_out, const float* w, float eps, float* xn,
                int8_t* xq, int8_t* xq2, float* xd, float* xs, int n, void* stream);

/* a = act(g) * u (u == NULL: act(g)), act = SiLU, or GELU in its tanh form when gelu != 0; n fp32 values
 * (n % 32 == 0) and their activation input.  Replaces: ggufengine/mmvq.py:959-966 (akt_q8) and its kernel
 * (:120-131). */
int qmv_act_q8(const float* g, const float* u, int gelu, float* a, int8_t* xq, int8_t* xq2, float* xd, float* xs,
               int n, void* stream);

#define QMV_OUT_F32 0
#define QMV_OUT_BF16 1
#define QMV_OUT_F16 2

/* Unpack n_values (a multiple of the block size) of block-format weights to dense values (out_dtype one of
 * QMV_OUT_*; out 16-byte aligned): the fp32 values of the reference's dequantiser bit for bit (the same
 * products and sums, each rounded), bf16 / fp16 rounded to nearest even from them.  Replaces:
 * ggufengine/mmvq.py:931-940 (entpacken, kernels aus_Q4_K / aus_Q6_K :496-534) for every format here, and
 * ggufengine/quant.py:484 (dequantize) on the GPU (the reference's PackedExperts.weights,
 * models/common.py:456-460, and QuantLinear.bf16_weight, qlinear.py:217). */
int qmv_unpack(int ggml_type, const uint8_t* w, long long n_values, void* out, int out_dtype, void* stream);

/* Programmatic dependent launch for the staged single-token kernels, the few-token tensor-core kernels,
 * the grouped MoE kernels and the activation producers (qmv_quant_q8, qmv_norm_q8, qmv_act_q8) (default
 * off): when on, each such kernel lets the next kernel
 * of the stream start early; a matvec streams its weights before the previous kernel has finished, and
 * every kernel reads its inputs and writes anything only after the previous kernel completed.  Turn it
 * on only when no kernel launched right before a matvec writes that matvec's weights.  Returns the old
 * value.
 * Replaces: nothing in the reference (its decoder relies on plain stream order, models/common.py:1185). */
int qmv_set_pdl(int enabled);

/* ---- decode chain ------------------------------------------------------------------------------- */

#define QMV_INPUT_RAW 0        /* x = a */
#define QMV_INPUT_RMSNORM 1    /* v = a (+ b, written to h_out when given); x = v * rsqrt(mean(v^2) + eps) * norm_w */
#define QMV_INPUT_SILU_MUL 2   /* x = silu(a) * b (b == NULL: silu(a)) */

/* One stage of a decode chain: 1..4 matrices of one format and row length n_in that read the same
 * input x, built by a fused producer from fp32 device vectors (a, b, norm_w: n_in values).
 * wait = 1: the stage reads outputs (y or h_out) of earlier stages, so all CTAs finish the previous
 * stage first.  Buffers the chain writes (y, h_out) must not be read by an earlier stage. */
typedef struct qmv_stage {
    int ggml_type;
    int n_jobs;
    const uint8_t* w[4];
    int n_out[4];
    float* y[4];
    int n_in;
    int input;
    const float* a;
    const float* b;
    const float* norm_w;
    float eps;
    float* h_out;
    int wait;
} qmv_stage;

/* A list of dependent single-token matvec stages (a decode step's projections with their RMS-norm and
 * SiLU-gate producers fused in) in one persistent, cooperative launch.  stages: host array of n_stages
 * (at most 128).  Shapes taken: Q4_K with n_in 4096 or 14336, Q6_K with n_in 4096 or 14336, Q8_0 with
 * n_in 4096 (others: QMV_ERR_SHAPE).  workspace: QMV_CHAIN_WORKSPACE_BYTES bytes of device memory,
 * 256-byte aligned (grid-barrier and group counters, cleared by the call on `stream`, and the
 * quantised activations); chains that run at the same time need separate workspaces.
 * A stage whose every input vector that the previous stage writes is one whole output of it has its
 * input quantised by the previous stage's CTAs as the 32-value groups complete; other stages quantise
 * their input at their start.  The quantised RMSNORM input is u = v * norm_w with the 1/rms factor
 * applied to its scales, so it can differ from quantising x itself by rounding.
 * Replaces: the reference's fused one-token layer step (ggufengine/models/baukasten.py:217-240:
 * norm_q8 -> mv(q,k,v) -> ... -> akt_q8 -> mv(down)) for its matvec and producer kernels
 * (mmvq.py:102-134, 852-865). */
#define QMV_CHAIN_WORKSPACE_BYTES 72704
int qmv_chain(const qmv_stage* stages, int n_stages, void* workspace, void* stream);

/* Bytes of workspace qmv_chain needs (QMV_CHAIN_WORKSPACE_BYTES).  Replaces: nothing in the reference. */
int64_t qmv_chain_workspace_bytes(void);

/* qmv_chain without a caller-provided workspace, for callers that cannot allocate device memory at
 * the call site: a runtime that owns every allocation up front (an arena or a caching allocator it
 * must not re-enter from inside a kernel-launch callback), or an FFI host (cgo, JNI, ctypes) with no
 * device allocator of its own.  The workspace is a fixed array in the library's device image
 * (QMV_CHAIN_WORKSPACE_BYTES); n_stages above QMV_CHAIN_NOALLOC_MAX_STAGES returns QMV_ERR_TOO_LARGE,
 * and nothing is allocated or freed by the call.  Its counters are cleared on `stream` before the
 * launch.  The first call on each device looks up the array's address with that device current
 * (module loading can happen then), so make that first call before any stream capture.  All calls on
 * one device share the one array: calls that overlap in time (other streams, other host threads) race
 * on it, so serialise them; use qmv_chain with a workspace each for concurrent chains.
 * Replaces: nothing — it has no counterpart in the reference (whose decoder allocates through torch). */
#define QMV_CHAIN_NOALLOC_MAX_STAGES 128
int qmv_chain_noalloc(const qmv_stage* stages, int n_stages, void* stream);

/* Values per unit of qmv_block_sums for a format (16 or 32; 0 for an unknown format). */
int qmv_unit_values(int ggml_type);

/* Test hook: the int32 sums of one token per (row, unit), unit = the values sharing one weight scale
 * and one activation scale (qmv_unit_values): s = sum code * xq, s2 = sum code * xq2, from the same
 * device code as qmv_mv.  s, s2: int32[n_out][n_in / unit], overwritten.
 * Replaces: nothing callable — it exposes the dp4a sums of ggufengine/mmvq.py:389-404 / :469-470. */
int qmv_block_sums(int ggml_type, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
                   int32_t* s, int32_t* s2, void* stream);

/* Reads (and with clear != 0 resets) the device status word; synchronises `stream`.  *out is host memory.
 * Replaces: nothing in the reference (its kernels have no device-side checks). */
int qmv_device_status(int clear, int* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* NEMICLI_QMV_H */
