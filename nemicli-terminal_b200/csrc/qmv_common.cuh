// Shared device helpers of the quantized matvec kernels (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace qmv {

// GGML type ids of the twenty-six formats (PQ2_0 = 142: the reference's id for the 128-value Q2_0 variant) (the GGUF type table; reference ggufengine/gguf.py:64-77)
enum : int {
    F_Q4_0 = 2, F_Q8_0 = 8, F_Q4_K = 12, F_Q5_K = 13, F_Q6_K = 14, F_IQ2_XXS = 16, F_IQ4_XS = 23, F_TQ2_0 = 35,
    F_MXFP4 = 39, F_IQ3_S = 21, F_IQ3_XXS = 18, F_Q4_1 = 3, F_Q5_0 = 6, F_Q5_1 = 7, F_IQ4_NL = 20,
    F_Q1_0 = 41, F_Q2_0 = 42, F_PQ2_0 = 142, F_Q3_K = 11, F_IQ2_XS = 17, F_IQ2_S = 22, F_Q2_K = 10, F_TQ1_0 = 34,
    F_IQ1_S = 19, F_IQ1_M = 29, F_PTQ1_0 = 143
};
// IQ1_S / IQ1_M: codebook entries of values in {-1, 0, +1} plus a +-1/8 delta
__host__ __device__ constexpr bool iq1_format(int f) { return f == F_IQ1_S || f == F_IQ1_M; }
// formats the staged single-token kernel takes (the rest run on the warp-per-row kernel)
__host__ __device__ constexpr bool staged_format(int f) { return f != F_TQ1_0 && !iq1_format(f) && f != F_PTQ1_0; }
// IQ2_XS / IQ2_S: 16-value scale groups, eight-magnitude codebook entries
__host__ __device__ constexpr bool iq2x_format(int f) { return f == F_IQ2_XS || f == F_IQ2_S; }
// the ternary / 1-bit formats with one scale per 64 or 128 values, taken in 32-value units
__host__ __device__ constexpr bool bits_format(int f) { return f == F_Q1_0 || f == F_Q2_0 || f == F_PQ2_0; }
// the 32-value block formats (one block per integer-sum unit)
__host__ __device__ constexpr bool b32_format(int f) {
    return f == F_Q4_0 || f == F_Q8_0 || f == F_MXFP4 || f == F_Q4_1 || f == F_Q5_0 || f == F_Q5_1 || f == F_IQ4_NL;
}

// status codes returned across the C ABI (include/nemicli_qmv.h)
enum : int {
    ST_OK = 0,
    ST_BAD_FORMAT = 1,
    ST_BAD_SHAPE = 2,
    ST_BAD_ALIGN = 3,
    ST_BAD_TOKENS = 4,
    ST_LAUNCH = 5,
    ST_NULL = 6,
    ST_DEVICE = 7,
};

// bits of the device-side status word (set by kernels, read with qmv_device_status)
enum : int { DEV_BAD_ADDRESS = 1 };
constexpr long long kPadSlot = -1;     // expert id of an unused slot: its output rows are zeros

constexpr int kWarpsPerBlock = 8;
constexpr int kMaxTokens = 8;           // tokens per launch of the dp4a kernels
constexpr float kInv254 = 1.0f / 254.0f;

__host__ __device__ constexpr int block_values(int f) {
    return b32_format(f) ? 32 : f == F_Q2_0 ? 64 : (f == F_Q1_0 || f == F_PQ2_0 || f == F_PTQ1_0) ? 128 : 256;
}
__host__ __device__ constexpr int block_bytes(int f) {
    return f == F_Q4_0 || f == F_IQ4_NL || f == F_Q1_0 || f == F_Q2_0 ? 18 : f == F_PQ2_0 ? 34 : f == F_IQ1_S ? 50 :
         f == F_IQ1_M ? 56 : f == F_PTQ1_0 ? 28 : f == F_Q3_K ? 110 : f == F_Q2_K ? 84 : f == F_TQ1_0 ? 54 : f == F_IQ2_XS ? 74 : f == F_IQ2_S ? 82 : f == F_Q4_1 ? 20 : f == F_Q5_0 ? 22 : f == F_Q5_1 ? 24 : f == F_Q8_0 ? 34 : f == F_Q4_K ? 144 : f == F_Q5_K ? 176 : f == F_Q6_K ? 210
         : f == F_IQ4_XS ? 136 : f == F_MXFP4 ? 17 : f == F_IQ3_S ? 110
         : f == F_IQ3_XXS ? 98 : 66;
}
// values per integer-sum unit (one weight scale and one activation scale)
__host__ __device__ constexpr int unit_values(int f) {
    return f == F_Q6_K || f == F_Q3_K || iq2x_format(f) || f == F_Q2_K || f == F_IQ1_M ? 16 : 32;
}
// Q3_K signed codes q2 - 4 (1 - hbit) of four values: 2-bit fields already in place (0x03 bytes), high bits
// in bit 0 of each byte
__device__ __forceinline__ uint32_t q3k_word(uint32_t q2, uint32_t h1) { return __vsub4(q2 | (h1 << 2), 0x04040404u); }

__host__ __device__ inline bool known_format(int f) {
    return f == F_Q4_0 || f == F_Q8_0 || f == F_Q4_K || f == F_Q5_K || f == F_Q6_K || f == F_IQ2_XXS || f == F_IQ4_XS ||
           f == F_TQ2_0 || f == F_MXFP4 || f == F_IQ3_S || f == F_IQ3_XXS || f == F_Q4_1 || f == F_Q5_0 ||
           f == F_Q5_1 || f == F_IQ4_NL || bits_format(f) || f == F_Q3_K || iq2x_format(f) || f == F_Q2_K || f == F_TQ1_0 ||
           iq1_format(f) || f == F_PTQ1_0;
}
// weight rows and blocks of the K-quant formats with 16-byte header words are read 16 bytes at a time;
// MXFP4's 17-byte blocks start at any byte, and their loads stay inside the tensor when it starts on a
// 4-byte boundary
__host__ __device__ constexpr int weight_align(int f) { return f == F_Q4_K || f == F_Q5_K ? 16 : f == F_MXFP4 ? 4 : 2;
}

// ---- loads --------------------------------------------------------------------------------------
// Weights are streamed once: non-coherent loads that do not allocate in L1.  Activations are
// re-read by every row and stay in L1 (__ldg).

__device__ __forceinline__ uint4 ldw16(const uint8_t* p) {            // 16-byte aligned
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldw4(const uint8_t* p) {          // 4-byte aligned
    uint32_t r;
    asm("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldw2(const uint8_t* p) {          // 2-byte aligned
    unsigned short r;
    asm("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(r) : "l"(p));
    return r;
}
__device__ __forceinline__ uint32_t ldw1(const uint8_t* p) {
    unsigned short r;
    asm("ld.global.nc.L1::no_allocate.u8 %0, [%1];" : "=h"(r) : "l"(p));
    return r & 0xFFu;
}
// 16 bytes at a 2-byte aligned address: aligned words, then funnel shifts.  Never reads past p + 16.
__device__ __forceinline__ uint4 ldw16_a2(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
    const uint32_t sh = uint32_t(a & 3) * 8u;                          // 0 or 16
    const uint32_t w0 = ldw4(b), w1 = ldw4(b + 4), w2 = ldw4(b + 8), w3 = ldw4(b + 12);
    const uint32_t w4 = sh ? ldw2(b + 16) : 0u;
    return make_uint4(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh),
                      __funnelshift_r(w2, w3, sh), __funnelshift_r(w3, w4, sh));
}
// 16 bytes at any address p, reading nothing outside [p & ~3, p + 16) (even p) or [p - 1, p + 16) (odd
// p: the byte before p is read, e.g. an MXFP4 block's scale before its 16 code bytes)
__device__ __forceinline__ uint4 ldw16_a1(const uint8_t* p) {
    if ((reinterpret_cast<uintptr_t>(p) & 1) == 0) return ldw16_a2(p);
    const uint4 a = ldw16_a2(p - 1);
    const uint32_t last = ldw1(p + 15);
    return make_uint4(__funnelshift_r(a.x, a.y, 8), __funnelshift_r(a.y, a.z, 8), __funnelshift_r(a.z, a.w, 8),
                      __funnelshift_r(a.w, last, 8));
}
__device__ __forceinline__ uint2 ldw8_a2(const uint8_t* p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
    const uint32_t sh = uint32_t(a & 3) * 8u;
    const uint32_t w0 = ldw4(b), w1 = ldw4(b + 4);
    const uint32_t w2 = sh ? ldw2(b + 8) : 0u;
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

__device__ __forceinline__ int4 ldx16(const int8_t* p) { return __ldg(reinterpret_cast<const int4*>(p)); }
__device__ __forceinline__ int2 ldx8(const int8_t* p) { return __ldg(reinterpret_cast<const int2*>(p)); }

__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half((unsigned short)bits)); }
__device__ __forceinline__ float bf2f(uint16_t bits) { return __uint_as_float(uint32_t(bits) << 16); }

__device__ __forceinline__ int dp4(uint32_t a, int b, int c) { return __dp4a(int(a), b, c); }

// 16-entry int8 codebooks of the formats, four entries per word: IQ4_XS (the reference's
// KVALUES_IQ4NL) and MXFP4 (e2m1 values doubled, KVALUES_MXFP4)
__host__ __device__ constexpr uint32_t kv4(int a, int b, int c, int d) {
    return uint32_t(uint8_t(a)) | (uint32_t(uint8_t(b)) << 8) | (uint32_t(uint8_t(c)) << 16) | (uint32_t(uint8_t(d)) << 24);
}
// the codebook values of four indices (one 0..15 index in each byte) as four int8 bytes: two byte
// permutes over the table's halves, the index's bit 3 picks the half
template <uint32_t T0, uint32_t T1, uint32_t T2, uint32_t T3>
__device__ __forceinline__ uint32_t lut16_bytes(uint32_t idx) {
    const uint32_t t = idx & 0x07070707u, v = t | (t >> 4);
    const uint32_t sel = (v & 0xFFu) | ((v >> 8) & 0xFF00u);
    const uint32_t lo = __byte_perm(T0, T1, sel), hi = __byte_perm(T2, T3, sel);
    const uint32_t m = ((idx >> 3) & 0x01010101u) * 0xFFu;
    return (lo & ~m) | (hi & m);
}
__device__ __forceinline__ uint32_t iq4nl_bytes(uint32_t idx) {
    return lut16_bytes<kv4(-127, -104, -83, -65), kv4(-49, -35, -22, -10), kv4(1, 13, 25, 38), kv4(53, 69, 89, 113)>(idx);
}
__device__ __forceinline__ uint32_t mxfp4_bytes(uint32_t idx) {
    return lut16_bytes<kv4(0, 1, 2, 3), kv4(4, 6, 8, 12), kv4(0, -1, -2, -3), kv4(-4, -6, -8, -12)>(idx);
}
// 4x4 byte transpose of 16 activation bytes: word s of the result holds values s, 4 + s, 8 + s, 12 + s
// (the order of Q2_0's 2-bit codes shifted by 2 s)
__device__ __forceinline__ int4 byte_transpose(int4 x) {
    const uint32_t t01 = __byte_perm(uint32_t(x.x), uint32_t(x.y), 0x5140), t23 = __byte_perm(uint32_t(x.z), uint32_t(x.w), 0x5140);
    const uint32_t u01 = __byte_perm(uint32_t(x.x), uint32_t(x.y), 0x7362), u23 = __byte_perm(uint32_t(x.z), uint32_t(x.w), 0x7362);
    return make_int4(int(__byte_perm(t01, t23, 0x5410)), int(__byte_perm(t01, t23, 0x7632)),
                     int(__byte_perm(u01, u23, 0x5410)), int(__byte_perm(u01, u23, 0x7632)));
}
// four bits to four bytes: bit j -> bit 0 of byte j
__device__ __forceinline__ uint32_t spread4(uint32_t s4) { return ((s4 & 15u) * 0x00204081u) & 0x01010101u; }
// byte masks of four sign bits (bit j set -> byte j = 0xFF)
__device__ __forceinline__ uint32_t sign4_mask(uint32_t s4) { return spread4(s4) * 0xFFu; }
// four magnitudes of {8, 25, 43} from four 2-bit level indices (one byte of a compact IQ2 codebook
// entry): each index to its byte, then 8 + 17 l + l / 2
__device__ __forceinline__ uint32_t iq2_mag4(uint32_t c4) {
    const uint32_t w = (c4 | (c4 << 6) | (c4 << 12) | (c4 << 18)) & 0x03030303u;
    return w * 17u + 0x08080808u + ((w >> 1) & 0x01010101u);
}
// MXFP4 block scale 2^(e-128) from its float bits (subnormal for e < 2), as the reference builds it
__device__ __forceinline__ float mxfp4_scale(uint32_t e) {
    return __uint_as_float(e < 2 ? (0x00200000u << e) : ((e - 1) << 23));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace qmv
