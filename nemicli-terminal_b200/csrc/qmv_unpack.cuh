// Unpacking GGUF blocks to dense values (the prefill side of the path: the reference unpacks a matrix for
// many input rows and multiplies it with cuBLAS, ggufengine/mmvq.py:496-534, 931-940, models/common.py:424).
//
// Every format's value is one of  A * c,  A * c + B,  A * c - B  with c a small exact integer code, A the
// scale of its 16- or 32-value group and B that group's offset, each rounded to fp32 in the order of the
// reference's dequantiser (ggufengine/quant.py, cited per format below).  The products and sums here use
// explicitly rounded intrinsics (no fused multiply-add), so the fp32 values are the reference's bit for bit
// and the bf16 / fp16 outputs are their round-to-nearest-even conversions.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "qmv_kernels.cuh"

namespace qmv {

__device__ __forceinline__ uint32_t ub(const uint8_t* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t u16le(const uint8_t* p) { return ub(p) | (ub(p + 1) << 8); }
__device__ __forceinline__ uint32_t u32le(const uint8_t* p) { return u16le(p) | (u16le(p + 2) << 16); }
__device__ __forceinline__ float hf(const uint8_t* p) { return h2f(u16le(p)); }
// 7 stored sign bits with the parity as the 8th (the IQ2 / IQ3 sign groups)
__device__ __forceinline__ uint32_t sign8(uint32_t s7) { return s7 | ((uint32_t(__popc(s7)) & 1u) << 7); }
__device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }

// 6-bit scale and minimum of sub-block j of a Q4_K / Q5_K header at s (quant.py:99-108)
__device__ __forceinline__ void scale_min6(const uint8_t* s, int j, int& sc, int& mn) {
    if (j < 4) {
        sc = int(ub(s + j) & 63);
        mn = int(ub(s + j + 4) & 63);
    } else {
        sc = int((ub(s + j + 4) & 15) | ((ub(s + j - 4) >> 6) << 4));
        mn = int((ub(s + j + 4) >> 4) | ((ub(s + j) >> 6) << 4));
    }
}

__device__ const int8_t kIq4nl[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
__device__ const int8_t kMxfp4[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

// values v0 .. v0 + 7 (v0 % 8 == 0) of the block at b
template <int FMT>
__device__ __forceinline__ void unpack8(const uint8_t* b, int v0, float (&o)[8]) {
    if constexpr (FMT == F_Q4_0) {                    // quant.py:60-64: d (q - 8)
        const float d = hf(b);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i, c = v < 16 ? int(ub(b + 2 + v) & 15) : int(ub(b + 2 + v - 16) >> 4);
            o[i] = mul(d, float(c - 8));
        }
    } else if constexpr (FMT == F_Q4_1) {             // quant.py:67-72: d q + m
        const float d = hf(b), m = hf(b + 2);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i, c = v < 16 ? int(ub(b + 4 + v) & 15) : int(ub(b + 4 + v - 16) >> 4);
            o[i] = __fadd_rn(mul(d, float(c)), m);
        }
    } else if constexpr (FMT == F_Q5_0 || FMT == F_Q5_1) {   // quant.py:75-95: d (q - 16), d q + m
        constexpr bool q51 = FMT == F_Q5_1;
        const float d = hf(b), m = q51 ? hf(b + 2) : 0.f;
        const uint32_t qh = u32le(b + (q51 ? 4 : 2));
        const uint8_t* qs = b + (q51 ? 8 : 6);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i;
            const int c = (v < 16 ? int(ub(qs + v) & 15) : int(ub(qs + v - 16) >> 4)) | int(((qh >> v) & 1u) << 4);
            o[i] = q51 ? __fadd_rn(mul(d, float(c)), m) : mul(d, float(c) - 16.0f);
        }
    } else if constexpr (FMT == F_Q8_0) {             // quant.py:46-50: d q
        const float d = hf(b);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = mul(d, float(int8_t(ub(b + 2 + v0 + i))));
    } else if constexpr (FMT == F_IQ4_NL || FMT == F_MXFP4) {   // quant.py:264, 390-401: codebook value x scale
        const float d = FMT == F_MXFP4 ? mxfp4_scale(ub(b)) : hf(b);
        const uint8_t* qs = b + (FMT == F_MXFP4 ? 1 : 2);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i, n = int((ub(qs + (v & 15)) >> (4 * (v >> 4))) & 15);
            o[i] = mul(float(FMT == F_MXFP4 ? kMxfp4[n] : kIq4nl[n]), d);
        }
    } else if constexpr (FMT == F_Q1_0) {             // quant.py:406-411: d (2 bit - 1)
        const float d = hf(b);
        const uint32_t bits = ub(b + 2 + v0 / 8);
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = mul(d, float(2 * int((bits >> i) & 1u) - 1));
    } else if constexpr (FMT == F_Q2_0 || FMT == F_PQ2_0) {     // quant.py:413-418: d (code - 1)
        const float d = hf(b);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i;
            o[i] = mul(d, float(int((ub(b + 2 + v / 4) >> (2 * (v % 4))) & 3)) - 1.0f);
        }
    } else if constexpr (FMT == F_TQ2_0) {            // quant.py:417-421: d (code - 1)
        const float d = hf(b + 64);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i, n = v >> 7, g = (v >> 5) & 3, m = v & 31;
            o[i] = mul(d, float(int((ub(b + 32 * n + m) >> (2 * g)) & 3)) - 1.0f);
        }
    } else if constexpr (FMT == F_TQ1_0) {            // quant.py:405-458: five trits per byte, d (trit - 1)
        const float d = hf(b + 52);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i;
            int byte, n;
            if (v < 160) { byte = v % 32; n = v / 32; }
            else if (v < 240) { byte = 32 + (v - 160) % 16; n = (v - 160) / 16; }
            else { byte = 48 + (v - 240) % 4; n = (v - 240) / 4; }
            const int pw = n == 0 ? 1 : n == 1 ? 3 : n == 2 ? 9 : n == 3 ? 27 : 81;
            const int t = int(((ub(b + byte) * uint32_t(pw)) & 255u) * 3u >> 8);
            o[i] = mul(d, float(t) - 1.0f);
        }
    } else if constexpr (FMT == F_Q2_K) {             // quant.py:284-292: (d sc) q - (dmin m), 16-value groups
        const int g = v0 / 16;
        const uint32_t s = ub(b + g);
        const float dl = mul(hf(b + 80), float(s & 15)), ml = mul(hf(b + 82), float(s >> 4));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i;
            const int c = int((ub(b + 16 + 32 * (v / 128) + v % 32) >> (2 * ((v % 128) / 32))) & 3);
            o[i] = __fsub_rn(mul(dl, float(c)), ml);
        }
    } else if constexpr (FMT == F_Q3_K) {             // quant.py:295-306: (d sc) q, signed 3-bit q, 16-value groups
        const int g = v0 / 16;
        const int lo = int((ub(b + 96 + g % 8) >> (4 * (g / 8))) & 15), hi = int((ub(b + 104 + g % 4) >> (2 * (g / 4))) & 3);
        const float dl = mul(hf(b + 108), float((lo | (hi << 4)) - 32));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i, n = v / 128, s = (v % 128) / 32, l = v % 32;
            const int q = int((ub(b + 32 + 32 * n + l) >> (2 * s)) & 3), h = int((ub(b + l) >> (v / 32)) & 1);
            o[i] = mul(dl, float(q - (h ? 0 : 4)));
        }
    } else if constexpr (FMT == F_Q4_K || FMT == F_Q5_K) {   // quant.py:111-137: (d sc) q - (dmin m)
        const int j = v0 / 32;
        int sc, mn;
        scale_min6(b + 4, j, sc, mn);
        const float a = mul(hf(b), float(sc)), m = mul(hf(b + 2), float(mn));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int l = (v0 + i) & 31;
            int q;
            if constexpr (FMT == F_Q4_K) q = int((ub(b + 16 + 32 * (j >> 1) + l) >> (4 * (j & 1))) & 15);
            else q = int((ub(b + 48 + 32 * (j >> 1) + l) >> (4 * (j & 1))) & 15) | int(((ub(b + 16 + l) >> j) & 1) << 4);
            o[i] = __fsub_rn(mul(a, float(q)), m);
        }
    } else if constexpr (FMT == F_Q6_K) {             // quant.py:140-159: (d sc) (q - 32), 16-value groups
        const int n = v0 >> 7, g = (v0 >> 5) & 3, l0 = v0 & 31;
        const float dl = mul(hf(b + 208), float(int8_t(ub(b + 192 + 8 * n + 2 * g + l0 / 16))));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int l = l0 + i;
            const int q = int((ub(b + 64 * n + 32 * (g & 1) + l) >> (4 * (g >> 1))) & 15) |
                          int(((ub(b + 128 + 32 * n + l) >> (2 * g)) & 3) << 4);
            o[i] = mul(dl, float(q - 32));
        }
    } else if constexpr (FMT == F_IQ4_XS) {           // quant.py:378-387: value x (d (ls - 32))
        const int ib = v0 / 32, j0 = v0 & 31;
        const int ls = int((ub(b + 4 + ib / 2) >> (4 * (ib & 1))) & 15) | int(((u16le(b + 2) >> (2 * ib)) & 3) << 4);
        const float dl = mul(hf(b), float(ls - 32));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int j = j0 + i;
            o[i] = mul(float(kIq4nl[(ub(b + 8 + 16 * ib + (j & 15)) >> (4 * (j >> 4))) & 15]), dl);
        }
    } else if constexpr (FMT == F_PTQ1_0) {           // quant.py:431-469: trits, d (trit - 1)
        const float d = hf(b + 26);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int v = v0 + i;
            int byte, n;
            if (v < 80) { byte = v % 16; n = v / 16; }
            else if (v < 120) { byte = 16 + (v - 80) % 8; n = (v - 80) / 8; }
            else { byte = 24 + (v - 120) % 2; n = (v - 120) / 2; }
            const int pw = n == 0 ? 1 : n == 1 ? 3 : n == 2 ? 9 : n == 3 ? 27 : 81;
            const int t = int(((ub(b + byte) * uint32_t(pw)) & 255u) * 3u >> 8);
            o[i] = mul(d, float(t) - 1.0f);
        }
    } else if constexpr (FMT == F_IQ1_S || FMT == F_IQ1_M) {   // quant.py:350-375: (d (2 s + 1)) (g + delta)
        const int e = v0 / 8;
        uint32_t idx, neg;
        float dl;
        if constexpr (FMT == F_IQ1_S) {
            const uint32_t qh = u16le(b + 34 + 2 * (e / 4));
            idx = ub(b + 2 + e) | (((qh >> (3 * (e % 4))) & 7u) << 8);
            neg = qh >> 15;
            dl = mul(hf(b), float(2 * int((qh >> 12) & 7u) + 1));
        } else {
            const uint32_t nib = (ub(b + 32 + e / 2) >> (4 * (e & 1))) & 15u;
            idx = ub(b + e) | ((nib & 7u) << 8);
            neg = nib >> 3;
            const uint32_t s0 = u16le(b + 48), s1 = u16le(b + 50), s2 = u16le(b + 52), s3 = u16le(b + 54);
            const uint32_t d16 = (s0 >> 12) | ((s1 >> 8) & 0xF0u) | ((s2 >> 4) & 0xF00u) | (s3 & 0xF000u);
            const int g = e / 2;
            const uint32_t sw = u16le(b + 48 + 2 * (g / 4));
            dl = mul(h2f(d16), float(2 * int((sw >> (3 * (g % 4))) & 7u) + 1));
        }
        const uint32_t code = kIq1sCodes[idx];
        const float delta = neg ? -0.125f : 0.125f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t f = (code >> (2 * i)) & 3u;
            o[i] = mul(dl, __fadd_rn(float(f == 3u ? -1 : int(f)), delta));
        }
    } else if constexpr (FMT == F_IQ2_XXS) {          // quant.py:235-245: value x (d (0.125 + 0.25 s))
        const int ib = v0 / 32, l = (v0 & 31) >> 3;
        const uint8_t* q = b + 2 + 8 * ib;
        const uint32_t aux1 = u32le(q + 4);
        const float db = mul(hf(b), 0.125f + 0.25f * float(aux1 >> 28));
        const uint32_t code = kIq2xxsCodes[ub(q + l)], s = sign8((aux1 >> (7 * l)) & 127u);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t lv = (code >> (2 * i)) & 3u;
            const int g = lv == 0 ? 8 : lv == 1 ? 25 : 43;
            o[i] = mul(float((s >> i) & 1u ? -g : g), db);
        }
    } else if constexpr (FMT == F_IQ2_XS || FMT == F_IQ2_S) {   // quant.py:248-260, 310-318
        const int k = v0 / 8, g16 = v0 / 16;
        uint32_t idx, s;
        if constexpr (FMT == F_IQ2_XS) {
            const uint32_t q = u16le(b + 2 + 2 * k);
            idx = q & 511u;
            s = sign8(q >> 9);
        } else {
            idx = ub(b + 2 + k) | (((ub(b + 66 + k / 4) >> (2 * (k % 4))) & 3u) << 8);
            s = ub(b + 34 + k);
        }
        const uint32_t code = FMT == F_IQ2_XS ? kIq2xsCodes[idx] : kIq2sCodes[idx];
        const uint32_t sc = (ub(b + (FMT == F_IQ2_XS ? 66 : 74) + g16 / 2) >> (4 * (g16 % 2))) & 15u;
        const float db = mul(hf(b), 0.125f + 0.25f * float(sc));
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t lv = (code >> (2 * i)) & 3u;
            const int g = lv == 0 ? 8 : lv == 1 ? 25 : 43;
            o[i] = mul(float((s >> i) & 1u ? -g : g), db);
        }
    } else if constexpr (FMT == F_IQ3_XXS) {          // quant.py:322-331: value x (d (0.25 + 0.5 s))
        const int ib = v0 / 32, t0 = v0 & 31;
        const uint32_t aux = u32le(b + 66 + 4 * ib);
        const float db = mul(hf(b), 0.25f + 0.5f * float(aux >> 28));
        const uint32_t s = sign8((aux >> (7 * (t0 / 8))) & 127u);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int t = t0 + i;
            const uint32_t lv = (kIq3xxsCodes[ub(b + 2 + 8 * ib + t / 4)] >> (3 * (t % 4))) & 7u;
            const int g = lv == 7u ? 62 : int(4 + 8 * lv);
            o[i] = mul(float((s >> (t % 8)) & 1u ? -g : g), db);
        }
    } else if constexpr (FMT == F_IQ3_S) {            // quant.py:334-346: value x (d (1 + 2 s))
        const int ib = v0 / 32, t0 = v0 & 31;
        const float db = mul(hf(b), float(1 + 2 * int((ub(b + 106 + ib / 2) >> (4 * (ib & 1))) & 15)));
        const uint32_t sg = ub(b + 74 + 4 * ib + t0 / 8);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int t = t0 + i;
            const uint32_t idx = ub(b + 2 + 8 * ib + t / 4) | (((ub(b + 66 + ib) >> (t / 4)) & 1u) << 8);
            const int g = int(2 * ((kIq3sCodes[idx] >> (3 * (t % 4))) & 7u) + 1);
            o[i] = mul(float((sg >> (t % 8)) & 1u ? -g : g), db);
        }
    }
}

// Thread t unpacks values [8 t, 8 t + 8) of the flat tensor.  OUT: 0 fp32, 1 bf16, 2 fp16.
template <int FMT, int OUT>
__global__ void __launch_bounds__(256) unpack_kernel(const uint8_t* __restrict__ w, void* __restrict__ out,
                                                     long long n_values) {
    constexpr int BV = block_values(FMT), BB = block_bytes(FMT);
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (8 * t >= n_values) return;
    const long long v = 8 * t, blk = v / BV;
    float o[8];
    unpack8<FMT>(w + blk * BB, int(v - blk * BV), o);
    if constexpr (OUT == 0) {
        float4* p = reinterpret_cast<float4*>(static_cast<float*>(out) + v);
        p[0] = make_float4(o[0], o[1], o[2], o[3]);
        p[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
        uint32_t h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            if constexpr (OUT == 1) {
                const __nv_bfloat162 x = __floats2bfloat162_rn(o[2 * i], o[2 * i + 1]);
                h[i] = *reinterpret_cast<const uint32_t*>(&x);
            } else {
                const __half2 x = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
                h[i] = *reinterpret_cast<const uint32_t*>(&x);
            }
        }
        *reinterpret_cast<uint4*>(static_cast<uint16_t*>(out) + v) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

}  // namespace qmv
