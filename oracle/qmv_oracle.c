/*
 * TEST INFRASTRUCTURE ONLY — the CPU oracle for the quantized matvec hot path.
 *
 * Only tests/, __graft_entry__.smoke() and bench.py (its cpu_baseline leg and `--impl reference`)
 * may load this library, and only as the checker or the timed CPU baseline.  The product path
 * (nemicli-terminal_b200/) never calls it and fails loudly without its CUDA library.
 *
 * What it restates (paths relative to the reference checkout):
 *   - activation quantisation into the two-stage int8 input ("Eingang"): ggufengine/mmvq.py:59-74
 *     (quant32) and :77-83 (quant_q8).  The reference compiles it with --use_fast_math; this
 *     restatement uses IEEE-rounded division and an explicit fused multiply-add so that it is
 *     reproducible bit for bit on the GPU (the kernels do the same).  Against the reference's
 *     fast-math build a quantised value can differ by one unit on a rounding tie.
 *   - the block dequantisers of ggufengine/quant.py for the twenty-three in-scope formats:
 *     deq_q4_0 :60, deq_q4_1 :67, deq_q5_0 :83, deq_q5_1 :90 (+ _q5_high_bits :74), deq_iq4_nl :264,
 *     deq_q1_0 :424, deq_q2_0 :410 (and PQ2_0, the same codes in 34-byte blocks of 128 values),
 *     deq_q2_k :284, deq_q3_k :295, TQ1_0 (_deq_trits :449 with trit_plan :430), deq_iq2_xs :310 and deq_iq2_s :248 (IQ2XS_GRID, IQ2S_GRID, compact in
 *     csrc/iq2xs_grid.inc, csrc/iq2s_grid.inc), deq_q8_0 :46, deq_q4_k :111 (+ _scale_min_k4 :99), deq_q5_k :123, deq_q6_k :140,
 *     deq_iq4_xs :378 (codebook KVALUES_IQ4NL, ggufengine/iqtabellen.py:7), deq_mxfp4 :394
 *     (KVALUES_MXFP4 :391, scale 2^(e-128) as the reference builds its float bits), deq_iq3_s :334
 *     (codebook ggufengine/iqtabellen.py IQ3S_GRID, kept compact in csrc/iq3s_grid.inc), deq_iq3_xxs
 *     :322 (IQ3XXS_GRID, compact in csrc/iq3xxs_grid.inc),
 *     deq_tq2_0 :417, deq_iq2_xxs :235 (codebook ggufengine/iqtabellen.py:11).  The operation
 *     order of each fp32 expression follows quant.py, so results are bit-identical.
 *   - the integer dot products of the reference's int8 path (ggufengine/mmvq.py:341-419 for
 *     Q4_K: per lane S = sum nibble*xq and S2 = sum nibble*xq2; :421-482 for Q6_K with signed
 *     q-32), and the same formula family for Q4_0, Q8_0, Q5_K, TQ2_0, IQ2_XXS, IQ3_XXS, IQ3_S, IQ4_XS, MXFP4
 *     (which the reference only has as float kernels, ggufengine/cudakern.py:315,307,379,432,187;
 *     Q5_K is Q4_K's sum with a 5-bit unsigned code, IQ4_XS and MXFP4 sum int8 codebook values).  Integer sums do not
 *     depend on how a kernel groups them, so the per-unit sums below are the exact values any
 *     correct kernel must produce from the same Eingang.
 *
 * Sum units (the values that share one weight scale and one activation scale):
 *   Q4_K, Q5_K, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, TQ2_0, IQ2_XXS, IQ3_XXS, IQ3_S, IQ4_NL, IQ4_XS, MXFP4: 32
 *   values (n_in/32 units).  Q4_1 and Q5_1 take their +m offset and Q5_0 its -16 d offset with xs.
 *   Q3_K, IQ2_XS, IQ2_S, Q2_K: 16 values (their scale groups; Q3_K codes q2 - 4 (1 - hbit), signed).
 *   Q2_K's minimum applies per 16 values, finer than xs: its offset multiplies the quantised input's own
 *   16-value sum, xd (sum xq + sum xq2 / 254), the same activation the code sums see.
 *   Q1_0, Q2_0, PQ2_0: 32-value units inside 128 / 64 / 128-value blocks; codes bit (weight 2 d, offset
 *   d: d (2 b - 1)) and q (offset d: d (q - 1)).
 *   Q6_K: 16.
 *   Q4_0 and TQ2_0 sums use the unsigned code (the -8 / -1 offset is applied with xs).
 *
 * Parity pins: the dequantisers are pinned to golden vectors generated from the reference's own
 * quant.dequantize (tests/golden/make_golden.py); the quantiser is pinned to the reference test's
 * invariants (tests/test_mmvq.py:123-127 there: xq*xd ~ x, + xq2*xd/254 ~ x, xs = sum x) and to
 * the formula; the integer path is pinned by an exact fp64 identity against the dequantised
 * weights.  No reference artefact pins the int32 sums themselves (the reference tests compare
 * floats only).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

enum { T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ4_XS = 23, T_TQ2_0 = 35, T_MXFP4 = 39,
       T_IQ3_S = 21, T_IQ3_XXS = 18, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_IQ4_NL = 20,
       T_Q1_0 = 41, T_Q2_0 = 42, T_PQ2_0 = 142, T_Q3_K = 11, T_IQ2_XS = 17, T_IQ2_S = 22, T_Q2_K = 10, T_TQ1_0 = 34,
       T_IQ1_S = 19, T_IQ1_M = 29, T_PTQ1_0 = 143 };

/* IQ1_S / IQ1_M codebook (ggufengine/iqtabellen.py:570, IQ1S_GRID): 2048 entries of eight values in
   {-1, 0, +1}, two bits each (00 = 0, 01 = +1, 11 = -1) */
static const uint16_t IQ1S_CODES[2048] = {
#include "../nemicli-terminal_b200/csrc/iq1s_grid.inc"
};
static int iq1s_value(int idx, int j) {
    const int f = (IQ1S_CODES[idx] >> (2 * j)) & 3;
    return f == 3 ? -1 : f;
}

static const uint16_t IQ2XS_CODES[512] = {
#include "../nemicli-terminal_b200/csrc/iq2xs_grid.inc"
};
static const uint16_t IQ2S_CODES[1024] = {
#include "../nemicli-terminal_b200/csrc/iq2s_grid.inc"
};

/* IQ4_XS codebook (part of the format: the reference's KVALUES_IQ4NL) */
static const int8_t IQ4NL_VALUES[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};
/* MXFP4 codebook: e2m1 values doubled (the reference's KVALUES_MXFP4), so the scale is 2^(e-128) */
static const int8_t MXFP4_VALUES[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};

/* 2^(e-128) from its float bits, subnormal for e < 2 (ggufengine/quant.py:397-399) */
static float mxfp4_scale(uint8_t e) {
    const uint32_t bits = e < 2 ? (0x00200000u << e) : ((uint32_t)(e - 1) << 23);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static const uint16_t IQ2XXS_CODES[256] = {
#include "../nemicli-terminal_b200/csrc/iq2xxs_grid.inc"
};
static const uint8_t IQ2XXS_LEVELS[3] = {8, 25, 43};
static const uint16_t IQ3S_CODES[512] = {
#include "../nemicli-terminal_b200/csrc/iq3s_grid.inc"
};

/* magnitude e (0..3) of IQ3_S codebook entry idx: 2 * (3-bit field) + 1 */
static int iq3s_mag(int idx, int e) { return 2 * ((IQ3S_CODES[idx] >> (3 * e)) & 7) + 1; }

/* signed value t (0..31) of sub-block ib of an IQ3_S block: d (f16), qs[64] at 2, qh[8] at 66 (bit 8 of
   the grid index of group 8 ib + j is bit j of qh[ib]), signs[32] at 74 (bit t % 8 of byte 4 ib + t / 8
   set: negative), scales[4] at 106 (quant.py:334-346) */
static int iq3s_value(const uint8_t* b, int ib, int t) {
    const int k = 8 * ib + t / 4;
    const int idx = b[2 + k] | (((b[66 + ib] >> (t / 4)) & 1) << 8);
    const int g = iq3s_mag(idx, t % 4);
    return ((b[74 + 4 * ib + t / 8] >> (t % 8)) & 1) ? -g : g;
}
static int iq3s_scale(const uint8_t* b, int ib) { return (b[106 + ib / 2] >> (4 * (ib & 1))) & 15; }

static const uint16_t IQ3XXS_CODES[256] = {
#include "../nemicli-terminal_b200/csrc/iq3xxs_grid.inc"
};
static const uint8_t IQ3XXS_LEVELS[8] = {4, 12, 20, 28, 36, 44, 52, 62};

/* ---- scalars -------------------------------------------------------------------------------- */

static float f16(const uint8_t* p) {
    /* IEEE binary16 (little endian) -> binary32, exact */
    uint32_t h = (uint32_t)p[0] | ((uint32_t)p[1] << 8);
    uint32_t sign = (h & 0x8000u) << 16, exp = (h >> 10) & 0x1F, man = h & 0x3FF, bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {                                  /* subnormal: renormalise */
            int e = -1;
            do { man <<= 1; ++e; } while (!(man & 0x400));
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float bf16(uint16_t u) {
    uint32_t bits = (uint32_t)u << 16;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

int orc_block_values(int fmt) {
    switch (fmt) {
    case T_Q4_0: case T_Q8_0: case T_MXFP4: case T_Q4_1: case T_Q5_0: case T_Q5_1: case T_IQ4_NL: return 32;
    case T_Q2_0: return 64;
    case T_Q1_0: case T_PQ2_0: return 128;
    case T_Q4_K: case T_Q5_K: case T_Q6_K: case T_IQ2_XXS: case T_IQ3_XXS: case T_IQ3_S: case T_IQ4_XS:
    case T_TQ2_0: case T_Q3_K: case T_IQ2_XS: case T_IQ2_S: case T_Q2_K: case T_TQ1_0: return 256;
    case T_IQ1_S: case T_IQ1_M: return 256;
    case T_PTQ1_0: return 128;
    }
    return 0;
}

int orc_block_bytes(int fmt) {
    switch (fmt) {
    case T_Q4_0: return 18;
    case T_Q4_1: return 20;
    case T_Q5_0: return 22;
    case T_Q5_1: return 24;
    case T_IQ4_NL: return 18;
    case T_Q1_0: case T_Q2_0: return 18;
    case T_PQ2_0: return 34;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_IQ2_XXS: return 66;
    case T_IQ4_XS: return 136;
    case T_IQ3_S: return 110;
    case T_IQ3_XXS: return 98;
    case T_Q3_K: return 110;
    case T_IQ2_XS: return 74;
    case T_IQ2_S: return 82;
    case T_Q2_K: return 84;
    case T_TQ1_0: return 54;
    case T_TQ2_0: return 66;
    case T_MXFP4: return 17;
    case T_IQ1_S: return 50;
    case T_IQ1_M: return 56;
    case T_PTQ1_0: return 28;
    }
    return 0;
}

/* values per integer-sum unit */
int orc_unit_values(int fmt) {
    return fmt == T_Q6_K || fmt == T_Q3_K || fmt == T_IQ2_XS || fmt == T_IQ2_S || fmt == T_Q2_K || fmt == T_IQ1_M ? 16 : 32;
}
/* TQ1_0 (54 B = qs[48], qh[4], d; quant.py:405-458): five trits per byte as a fixed-point fraction, trit n of
   byte v = ((v 3^n) mod 256) 3 >> 8.  Value j < 160: byte j % 32, n = j / 32; j < 240: byte 32 + (j - 160) % 16,
   n = (j - 160) / 16; else byte 48 + (j - 240) % 4, n = (j - 240) / 4.  The code is the trit (offset d xs). */
static int tq1_trit(const uint8_t* b, int v) {
    static const int pw[5] = {1, 3, 9, 27, 81};
    int byte, n;
    if (v < 160) { byte = v % 32; n = v / 32; }
    else if (v < 240) { byte = 32 + (v - 160) % 16; n = (v - 160) / 16; }
    else { byte = 48 + (v - 240) % 4; n = (v - 240) / 4; }
    return (((b[byte] * pw[n]) & 255) * 3) >> 8;
}
/* PTQ1_0 (28 B = qs[24], qh[2], d; quant.py:431-469, trit_plan(24, 2)): values 0..79 are trit n = j / 16
   of byte j % 16, 80..119 trit n = (j - 80) / 8 of byte 16 + (j - 80) % 8, 120..127 trit n = (j - 120) / 2 of
   qh byte 24 + (j - 120) % 2.  The code is the trit (offset d xs). */
static int ptq1_trit(const uint8_t* b, int v) {
    static const int pw[5] = {1, 3, 9, 27, 81};
    int byte, n;
    if (v < 80) { byte = v % 16; n = v / 16; }
    else if (v < 120) { byte = 16 + (v - 80) % 8; n = (v - 80) / 8; }
    else { byte = 24 + (v - 120) % 2; n = (v - 120) / 2; }
    return (((b[byte] * pw[n]) & 255) * 3) >> 8;
}
/* IQ1_S (50 B = d, qs[32], qh[8] u16; quant.py:350-360): sub-block ib's u16 qh holds three high index bits
   per entry (bits 3l..3l+2), a 3-bit scale (bits 12..14) and the sign of its delta (bit 15).
   IQ1_M (56 B = qs[32], qh[16] (a nibble per entry: three high index bits and the delta sign), scales
   u16[4] (3-bit scale of each 16-value group in bits 0..11, d's four nibbles in bits 12..15);
   quant.py:363-375).  Value = dl (grid + delta), dl = d (2 s + 1), delta = +-1/8: the integer code is
   8 grid +- 1 with weight scale dl / 8. */
static int iq1_entry(const uint8_t* b, int fmt, int e, int* neg) {
    if (fmt == T_IQ1_S) {
        const int qh = b[34 + 2 * (e / 4)] | (b[35 + 2 * (e / 4)] << 8);
        *neg = (qh >> 15) & 1;
        return b[2 + e] | (((qh >> (3 * (e % 4))) & 7) << 8);
    }
    const int nib = (b[32 + e / 2] >> (4 * (e & 1))) & 15;
    *neg = nib >> 3;
    return b[e] | ((nib & 7) << 8);
}
static float iq1m_d(const uint8_t* b) {
    int sc[4];
    for (int i = 0; i < 4; ++i) sc[i] = b[48 + 2 * i] | (b[49 + 2 * i] << 8);
    const int d16 = (sc[0] >> 12) | ((sc[1] >> 8) & 0xF0) | ((sc[2] >> 4) & 0xF00) | (sc[3] & 0xF000);
    const uint8_t h[2] = {(uint8_t)(d16 & 0xFF), (uint8_t)(d16 >> 8)};
    return f16(h);
}
static int iq1_scale(const uint8_t* b, int fmt, int g) {   /* 3-bit scale: sub-block g (IQ1_S), 16-value group g (IQ1_M) */
    if (fmt == T_IQ1_S) return ((b[34 + 2 * g] | (b[35 + 2 * g] << 8)) >> 12) & 7;
    const int sc = b[48 + 2 * (g / 4)] | (b[49 + 2 * (g / 4)] << 8);
    return (sc >> (3 * (g % 4))) & 7;
}

/* Q2_K (84 B = scales[16] (scale nibble, min nibble), qs[64], d, dmin; quant.py:284-292): code of value v */
static int q2k_code(const uint8_t* b, int v) { return (b[16 + 32 * (v / 128) + v % 32] >> (2 * ((v % 128) / 32))) & 3; }

/* Q3_K (110 B = hmask[32], qs[64], scales[12], d; quant.py:295-306): scale group i (16 values) and the
   signed code of value v (0..255) */
static int q3k_scale(const uint8_t* b, int i) {
    const int lo = (b[96 + i % 8] >> (4 * (i / 8))) & 15, hi = (b[104 + i % 4] >> (2 * (i / 4))) & 3;
    return (lo | (hi << 4)) - 32;
}
/* IQ2_XS (74 B = d, u16 qs[32], scales[8]; quant.py:310-318): entry k (8 values) has codebook index
   bits 0..8 and a 7-bit sign index (parity gives the 8th sign) in bits 9..15.  IQ2_S (82 B = d, qs[32],
   signs[32], qh[8], scales[8]; quant.py:248-260): entry k has index qs[k] | bits 2 (k % 4).. of qh[k / 4]
   << 8 and sign byte signs[k].  Both: 4-bit scale of 16-value group i = nibble i % 2 of scales[i / 2],
   weight scale d (0.125 + 0.25 s). */
static uint32_t ksign8(uint32_t s7);
static int iq2xs_value(const uint8_t* b, int fmt, int v) {
    const int k = v / 8, j = v % 8;
    int idx, s8;
    if (fmt == T_IQ2_XS) {
        const int q = b[2 + 2 * k] | (b[3 + 2 * k] << 8);
        idx = q & 511;
        s8 = (int)ksign8((uint32_t)(q >> 9));
    } else {
        idx = b[2 + k] | (((b[66 + k / 4] >> (2 * (k % 4))) & 3) << 8);
        s8 = b[34 + k];
    }
    const int code = fmt == T_IQ2_XS ? IQ2XS_CODES[idx] : IQ2S_CODES[idx];
    const int g = IQ2XXS_LEVELS[(code >> (2 * j)) & 3];
    return (s8 >> j) & 1 ? -g : g;
}
static int iq2xs_scale(const uint8_t* b, int fmt, int i) {
    return (b[(fmt == T_IQ2_XS ? 66 : 74) + i / 2] >> (4 * (i % 2))) & 15;
}
static int q3k_code(const uint8_t* b, int v) {
    const int n = v / 128, s = (v % 128) / 32, l = v % 32;
    const int q = (b[32 + 32 * n + l] >> (2 * s)) & 3, h = (b[l] >> (v / 32)) & 1;
    return q - (h ? 0 : 4);
}

/* ---- activation quantisation (mmvq.py:59-83) ----------------------------------------------- */

/* Sum of 32 values in the order of a warp butterfly (xor 16, 8, 4, 2, 1): the order the GPU uses. */
static float butterfly_sum32(const float* v) {
    float a[16], b[8], c[4], d[2];
    for (int i = 0; i < 16; ++i) a[i] = v[i] + v[i + 16];
    for (int i = 0; i < 8; ++i) b[i] = a[i] + a[i + 8];
    for (int i = 0; i < 4; ++i) c[i] = b[i] + b[i + 4];
    for (int i = 0; i < 2; ++i) d[i] = c[i] + c[i + 2];
    return d[0] + d[1];
}

static int clamp127(int v) { return v < -127 ? -127 : (v > 127 ? 127 : v); }

/* x: n values, fp32 (x_is_f32) or bf16; n % 32 == 0 */
void orc_quant_q8(const void* x, int x_is_f32, long long n, int8_t* xq, int8_t* xq2, float* xd, float* xs) {
    for (long long g = 0; g < n / 32; ++g) {
        float v[32], amax = 0.f;
        for (int i = 0; i < 32; ++i) {
            v[i] = x_is_f32 ? ((const float*)x)[32 * g + i] : bf16(((const uint16_t*)x)[32 * g + i]);
            float a = fabsf(v[i]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / 127.0f;
        const float d2 = d / 254.0f;
        for (int i = 0; i < 32; ++i) {
            int q = 0, q2 = 0;
            if (d > 0.f) {
                q = (int)rintf(v[i] / d);
                const float r = fmaf(-(float)q, d, v[i]);
                q2 = clamp127((int)rintf(r / d2));
            }
            xq[32 * g + i] = (int8_t)q;
            xq2[32 * g + i] = (int8_t)q2;
        }
        xd[g] = d;
        xs[g] = butterfly_sum32(v);
    }
}

/* ---- dequantisation (quant.py) ------------------------------------------------------------- */

static void scale_min_k4(const uint8_t* s, int* sc, int* mn) {   /* quant.py:99-108 */
    for (int j = 0; j < 4; ++j) {
        sc[j] = s[j] & 63;
        mn[j] = s[j + 4] & 63;
        sc[j + 4] = (s[j + 8] & 15) | ((s[j] >> 6) << 4);
        mn[j + 4] = (s[j + 8] >> 4) | ((s[j + 4] >> 6) << 4);
    }
}

static void iq2xxs_entry(int idx, uint8_t out[8]) {
    for (int j = 0; j < 8; ++j) out[j] = IQ2XXS_LEVELS[(IQ2XXS_CODES[idx] >> (2 * j)) & 3];
}

static uint32_t ksign8(uint32_t s7) {   /* 7 stored sign bits + parity as the 8th */
    return s7 | ((uint32_t)(__builtin_popcount(s7) & 1) << 7);
}

/* signed value of element e (0..31) of sub-block ib of an IQ2_XXS block, without the scale */
static int iq2xxs_value(const uint8_t* b, int ib, int e) {
    const uint8_t* q = b + 2 + 8 * ib;
    const uint32_t aux1 = rd32(q + 4);
    const int l = e >> 3, j = e & 7;
    uint8_t g[8];
    iq2xxs_entry(q[l], g);
    const uint32_t s = ksign8((aux1 >> (7 * l)) & 127);
    return (s >> j) & 1 ? -(int)g[j] : (int)g[j];
}

/* signed value t (0..31) of sub-block ib of an IQ3_XXS block: d (f16), qs[64] at 2 (codebook index of
   values 4k..4k+3 of the sub-block at qs[8 ib + k]), aux u32[8] at 66: four 7-bit sign groups of 8 values
   (parity gives the 8th sign) and a 4-bit scale in bits 28..31 (quant.py:322-331) */
static int iq3xxs_value(const uint8_t* b, int ib, int t) {
    const uint32_t aux = rd32(b + 66 + 4 * ib);
    const int g = IQ3XXS_LEVELS[(IQ3XXS_CODES[b[2 + 8 * ib + t / 4]] >> (3 * (t % 4))) & 7];
    const uint32_t s = ksign8((aux >> (7 * (t / 8))) & 127);
    return (s >> (t % 8)) & 1 ? -g : g;
}

int orc_dequant(int fmt, const uint8_t* raw, long long n_values, float* out) {
    const int bv = orc_block_values(fmt), bb = orc_block_bytes(fmt);
    if (!bv || n_values % bv) return 2;
    for (long long blk = 0; blk < n_values / bv; ++blk) {
        const uint8_t* b = raw + blk * bb;
        float* o = out + blk * bv;
        switch (fmt) {
        case T_Q4_0: {
            const float d = f16(b);
            for (int i = 0; i < 16; ++i) {
                o[i] = d * (float)((b[2 + i] & 15) - 8);
                o[i + 16] = d * (float)((b[2 + i] >> 4) - 8);
            }
            break;
        }
        case T_Q8_0: {
            const float d = f16(b);
            for (int i = 0; i < 32; ++i) o[i] = d * (float)(int8_t)b[2 + i];
            break;
        }
        case T_Q4_1: {           /* d, m, 16 B nibbles: d q + m */
            const float d = f16(b), m = f16(b + 2);
            for (int i = 0; i < 16; ++i) {
                o[i] = d * (float)(b[4 + i] & 15) + m;
                o[i + 16] = d * (float)(b[4 + i] >> 4) + m;
            }
            break;
        }
        case T_Q5_0: case T_Q5_1: {   /* d (, m), qh u32: bit j is bit 4 of value j; 16 B nibbles */
            const int q51 = fmt == T_Q5_1;
            const float d = f16(b), m = q51 ? f16(b + 2) : 0.f;
            const uint32_t qh = rd32(b + (q51 ? 4 : 2));
            const uint8_t* qs = b + (q51 ? 8 : 6);
            for (int i = 0; i < 16; ++i) {
                const int lo = (qs[i] & 15) | (int)(((qh >> i) & 1) << 4);
                const int hi = (qs[i] >> 4) | (int)(((qh >> (i + 16)) & 1) << 4);
                if (q51) {
                    o[i] = d * (float)lo + m;
                    o[i + 16] = d * (float)hi + m;
                } else {
                    o[i] = d * ((float)lo - 16.0f);
                    o[i + 16] = d * ((float)hi - 16.0f);
                }
            }
            break;
        }
        case T_TQ1_0: {
            const float d = f16(b + 52);
            for (int j = 0; j < 256; ++j) o[j] = d * ((float)tq1_trit(b, j) - 1.0f);
            break;
        }
        case T_Q2_K: {
            const float d = f16(b + 80), dmin = f16(b + 82);
            for (int i = 0; i < 16; ++i) {
                const float dl = d * (float)(b[i] & 15), ml = dmin * (float)(b[i] >> 4);
                for (int l = 0; l < 16; ++l) o[16 * i + l] = dl * (float)q2k_code(b, 16 * i + l) - ml;
            }
            break;
        }
        case T_IQ2_XS: case T_IQ2_S: {
            const float d = f16(b);
            for (int i = 0; i < 16; ++i) {
                const float db = d * (0.125f + 0.25f * (float)iq2xs_scale(b, fmt, i));
                for (int l = 0; l < 16; ++l) o[16 * i + l] = (float)iq2xs_value(b, fmt, 16 * i + l) * db;
            }
            break;
        }
        case T_Q3_K: {
            const float d = f16(b + 108);
            for (int i = 0; i < 16; ++i) {
                const float dl = d * (float)q3k_scale(b, i);
                for (int l = 0; l < 16; ++l) o[16 * i + l] = dl * (float)q3k_code(b, 16 * i + l);
            }
            break;
        }
        case T_IQ1_S: {
            const float d = f16(b);
            for (int ib = 0; ib < 8; ++ib) {
                const float dl = d * (float)(2 * iq1_scale(b, T_IQ1_S, ib) + 1);
                for (int l = 0; l < 4; ++l) {
                    int neg;
                    const int idx = iq1_entry(b, T_IQ1_S, 4 * ib + l, &neg);
                    for (int j = 0; j < 8; ++j) o[32 * ib + 8 * l + j] = dl * ((float)iq1s_value(idx, j) + (neg ? -0.125f : 0.125f));
                }
            }
            break;
        }
        case T_IQ1_M: {
            const float d = iq1m_d(b);
            for (int e = 0; e < 32; ++e) {
                const float dl = d * (float)(2 * iq1_scale(b, T_IQ1_M, e / 2) + 1);
                int neg;
                const int idx = iq1_entry(b, T_IQ1_M, e, &neg);
                for (int j = 0; j < 8; ++j) o[8 * e + j] = ((float)iq1s_value(idx, j) + (neg ? -0.125f : 0.125f)) * dl;
            }
            break;
        }
        case T_PTQ1_0: {
            const float d = f16(b + 26);
            for (int j = 0; j < 128; ++j) o[j] = d * ((float)ptq1_trit(b, j) - 1.0f);
            break;
        }
        case T_Q2_0: case T_PQ2_0: {  /* d, then 2-bit codes: value j at bits 2 (j % 4) of byte j / 4 */
            const float d = f16(b);
            for (int j = 0; j < bv; ++j) o[j] = d * ((float)((b[2 + j / 4] >> (2 * (j % 4))) & 3) - 1.0f);
            break;
        }
        case T_Q1_0: {           /* d, then bits: value j = bit j % 8 of byte j / 8, d (2 b - 1) */
            const float d = f16(b);
            for (int j = 0; j < 128; ++j) o[j] = d * (2.0f * (float)((b[2 + j / 8] >> (j % 8)) & 1) - 1.0f);
            break;
        }
        case T_IQ4_NL: {         /* d, 16 B: byte j holds codebook indices of values j (low) and 16 + j */
            const float d = f16(b);
            for (int j = 0; j < 16; ++j) {
                o[j] = (float)IQ4NL_VALUES[b[2 + j] & 15] * d;
                o[j + 16] = (float)IQ4NL_VALUES[b[2 + j] >> 4] * d;
            }
            break;
        }
        case T_Q4_K: {
            const float d = f16(b), dmin = f16(b + 2);
            int sc[8], mn[8];
            scale_min_k4(b + 4, sc, mn);
            for (int j = 0; j < 8; ++j) {
                const float a = d * (float)sc[j], m = dmin * (float)mn[j];
                for (int i = 0; i < 32; ++i) {
                    const int q = (b[16 + 32 * (j >> 1) + i] >> (4 * (j & 1))) & 15;
                    o[32 * j + i] = a * (float)q - m;
                }
            }
            break;
        }
        case T_Q5_K: {
            /* d, dmin, 12 B scales/mins as Q4_K, qh[32] at 16, qs[128] at 48: sub-block j value i is the
               nibble (j odd: high) of qs[32 (j/2) + i] with bit j of qh[i] as bit 4 (quant.py:123-137) */
            const float d = f16(b), dmin = f16(b + 2);
            int sc[8], mn[8];
            scale_min_k4(b + 4, sc, mn);
            for (int j = 0; j < 8; ++j) {
                const float a = d * (float)sc[j], m = dmin * (float)mn[j];
                for (int i = 0; i < 32; ++i) {
                    const int q = ((b[48 + 32 * (j >> 1) + i] >> (4 * (j & 1))) & 15) | (((b[16 + i] >> j) & 1) << 4);
                    o[32 * j + i] = a * (float)q - m;
                }
            }
            break;
        }
        case T_Q6_K: {
            const uint8_t* ql = b;
            const uint8_t* qh = b + 128;
            const int8_t* sc = (const int8_t*)(b + 192);
            const float d = f16(b + 208);
            for (int n = 0; n < 2; ++n)
                for (int g = 0; g < 4; ++g)
                    for (int l = 0; l < 32; ++l) {
                        const int q = ((ql[64 * n + 32 * (g & 1) + l] >> (4 * (g >> 1))) & 15)
                                      | (((qh[32 * n + l] >> (2 * g)) & 3) << 4);
                        o[128 * n + 32 * g + l] = d * (float)sc[8 * n + 2 * g + l / 16] * (float)(q - 32);
                    }
            break;
        }
        case T_IQ4_XS: {
            /* d (f16), scales_h (u16) at 2, scales_l[4] at 4, qs[128] at 8: sub-block ib's 6-bit scale is
               nibble ib%2 of scales_l[ib/2] with bits 2ib..2ib+1 of scales_h on top; qs[16 ib + j] holds
               values j (low nibble) and 16 + j (high) as codebook indices (quant.py:378-387) */
            const float d = f16(b);
            const int sh = b[2] | (b[3] << 8);
            for (int ib = 0; ib < 8; ++ib) {
                const int ls = ((b[4 + ib / 2] >> (4 * (ib & 1))) & 15) | (((sh >> (2 * ib)) & 3) << 4);
                const float dl = d * (float)(ls - 32);
                for (int j = 0; j < 16; ++j) {
                    o[32 * ib + j] = (float)IQ4NL_VALUES[b[8 + 16 * ib + j] & 15] * dl;
                    o[32 * ib + 16 + j] = (float)IQ4NL_VALUES[b[8 + 16 * ib + j] >> 4] * dl;
                }
            }
            break;
        }
        case T_IQ3_XXS: {
            const float d = f16(b);
            for (int ib = 0; ib < 8; ++ib) {
                const float db = d * (0.25f + 0.5f * (float)(rd32(b + 66 + 4 * ib) >> 28));
                for (int t = 0; t < 32; ++t) o[32 * ib + t] = (float)iq3xxs_value(b, ib, t) * db;
            }
            break;
        }
        case T_IQ3_S: {
            const float d = f16(b);
            for (int ib = 0; ib < 8; ++ib) {
                const float db = d * (float)(1 + 2 * iq3s_scale(b, ib));
                for (int t = 0; t < 32; ++t) o[32 * ib + t] = (float)iq3s_value(b, ib, t) * db;
            }
            break;
        }
        case T_MXFP4: {
            /* e (E8M0) then 16 bytes: byte j holds values j (low nibble) and 16 + j (high) */
            const float d = mxfp4_scale(b[0]);
            for (int j = 0; j < 16; ++j) {
                o[j] = (float)MXFP4_VALUES[b[1 + j] & 15] * d;
                o[16 + j] = (float)MXFP4_VALUES[b[1 + j] >> 4] * d;
            }
            break;
        }
        case T_TQ2_0: {
            const float d = f16(b + 64);
            for (int n = 0; n < 2; ++n)
                for (int g = 0; g < 4; ++g)
                    for (int m = 0; m < 32; ++m)
                        o[128 * n + 32 * g + m] = d * (float)(((b[32 * n + m] >> (2 * g)) & 3) - 1);
            break;
        }
        case T_IQ2_XXS: {
            const float d = f16(b);
            for (int ib = 0; ib < 8; ++ib) {
                const uint32_t aux1 = rd32(b + 2 + 8 * ib + 4);
                const float db = d * (0.125f + 0.25f * (float)(aux1 >> 28));
                for (int e = 0; e < 32; ++e) o[32 * ib + e] = (float)iq2xxs_value(b, ib, e) * db;
            }
            break;
        }
        default:
            return 1;
        }
    }
    return 0;
}

/* ---- integer sums and the epilogue --------------------------------------------------------- */

/* integer weight code of value v (0 <= v < block values) of block b, as used by the dot product */
static int code_of(int fmt, const uint8_t* b, int v) {
    switch (fmt) {
    case T_Q4_0: return v < 16 ? (b[2 + v] & 15) : (b[2 + v - 16] >> 4);
    case T_Q8_0: return (int8_t)b[2 + v];
    case T_Q4_1: return v < 16 ? (b[4 + v] & 15) : (b[4 + v - 16] >> 4);
    case T_Q5_0: case T_Q5_1: {
        const int q51 = fmt == T_Q5_1;
        const uint32_t qh = rd32(b + (q51 ? 4 : 2));
        const uint8_t* qs = b + (q51 ? 8 : 6);
        return (v < 16 ? (qs[v] & 15) : (qs[v - 16] >> 4)) | (int)(((qh >> v) & 1) << 4);
    }
    case T_IQ4_NL: return IQ4NL_VALUES[(b[2 + (v & 15)] >> (4 * (v >> 4))) & 15];
    case T_Q2_0: case T_PQ2_0: return (b[2 + v / 4] >> (2 * (v % 4))) & 3;
    case T_Q1_0: return (b[2 + v / 8] >> (v % 8)) & 1;
    case T_Q3_K: return q3k_code(b, v);
    case T_Q2_K: return q2k_code(b, v);
    case T_TQ1_0: return tq1_trit(b, v);
    case T_PTQ1_0: return ptq1_trit(b, v);
    case T_IQ1_S: case T_IQ1_M: {
        int neg;
        const int idx = iq1_entry(b, fmt, v / 8, &neg);
        return 8 * iq1s_value(idx, v % 8) + (neg ? -1 : 1);
    }
    case T_IQ2_XS: case T_IQ2_S: return iq2xs_value(b, fmt, v);
    case T_Q4_K: { const int j = v >> 5, i = v & 31; return (b[16 + 32 * (j >> 1) + i] >> (4 * (j & 1))) & 15; }
    case T_Q5_K: {
        const int j = v >> 5, i = v & 31;
        return ((b[48 + 32 * (j >> 1) + i] >> (4 * (j & 1))) & 15) | (((b[16 + i] >> j) & 1) << 4);
    }
    case T_Q6_K: {
        const int n = v >> 7, g = (v >> 5) & 3, l = v & 31;
        const int q = ((b[64 * n + 32 * (g & 1) + l] >> (4 * (g >> 1))) & 15) | (((b[128 + 32 * n + l] >> (2 * g)) & 3) << 4);
        return q - 32;
    }
    case T_TQ2_0: { const int n = v >> 7, g = (v >> 5) & 3, m = v & 31; return (b[32 * n + m] >> (2 * g)) & 3; }
    case T_IQ2_XXS: return iq2xxs_value(b, v >> 5, v & 31);
    case T_MXFP4: return MXFP4_VALUES[(b[1 + (v & 15)] >> (4 * (v >> 4))) & 15];
    case T_IQ3_S: return iq3s_value(b, v >> 5, v & 31);
    case T_IQ3_XXS: return iq3xxs_value(b, v >> 5, v & 31);
    case T_IQ4_XS: {
        const int ib = v >> 5, j = v & 31;
        return IQ4NL_VALUES[(b[8 + 16 * ib + (j & 15)] >> (4 * (j >> 4))) & 15];
    }
    }
    return 0;
}

/* s, s2: [n_out][n_in / unit] int32 sums of code * xq and code * xq2 (one token) */
int orc_block_sums(int fmt, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
                   int32_t* s, int32_t* s2) {
    const int bv = orc_block_values(fmt), bb = orc_block_bytes(fmt), uv = orc_unit_values(fmt);
    if (!bv || n_in % bv) return 2;
    const long long row_bytes = (long long)(n_in / bv) * bb;
    const int units = n_in / uv;
    for (int r = 0; r < n_out; ++r)
        for (int u = 0; u < units; ++u) {
            int32_t a = 0, a2 = 0;
            for (int i = 0; i < uv; ++i) {
                const int v = u * uv + i;
                const int c = code_of(fmt, w + r * row_bytes + (long long)(v / bv) * bb, v % bv);
                a += c * xq[v];
                a2 += c * xq2[v];
            }
            s[(long long)r * units + u] = a;
            s2[(long long)r * units + u] = a2;
        }
    return 0;
}

/* weight scale (multiplies xd*(S + S2/254)) and offset (multiplies xs) of unit u of block b */
static void unit_scales(int fmt, const uint8_t* b, int u, double* wscale, double* offs) {
    switch (fmt) {
    case T_Q4_0: *wscale = f16(b); *offs = 8.0 * f16(b); return;
    case T_Q8_0: *wscale = f16(b); *offs = 0.0; return;
    case T_Q4_1: case T_Q5_1: *wscale = f16(b); *offs = -(double)f16(b + 2); return;
    case T_Q5_0: *wscale = f16(b); *offs = 16.0 * f16(b); return;
    case T_IQ4_NL: *wscale = f16(b); *offs = 0.0; return;
    case T_Q2_0: case T_PQ2_0: *wscale = f16(b); *offs = f16(b); return;
    case T_Q1_0: *wscale = 2.0 * f16(b); *offs = f16(b); return;
    case T_Q3_K: *wscale = (double)f16(b + 108) * (double)q3k_scale(b, u); *offs = 0.0; return;
    case T_TQ1_0: *wscale = f16(b + 52); *offs = f16(b + 52); return;
    case T_PTQ1_0: *wscale = f16(b + 26); *offs = f16(b + 26); return;
    case T_IQ1_S: *wscale = (double)f16(b) * (double)(2 * iq1_scale(b, T_IQ1_S, u) + 1) / 8.0; *offs = 0.0; return;
    case T_IQ1_M: *wscale = (double)iq1m_d(b) * (double)(2 * iq1_scale(b, T_IQ1_M, u) + 1) / 8.0; *offs = 0.0; return;
    case T_Q2_K: *wscale = (double)f16(b + 80) * (double)(b[u] & 15); *offs = (double)f16(b + 82) * (double)(b[u] >> 4); return;
    case T_IQ2_XS: case T_IQ2_S:
        *wscale = (double)f16(b) * (0.125 + 0.25 * (double)iq2xs_scale(b, fmt, u));
        *offs = 0.0;
        return;
    case T_Q4_K: case T_Q5_K: {
        int sc[8], mn[8];
        scale_min_k4(b + 4, sc, mn);
        *wscale = (double)f16(b) * sc[u];
        *offs = (double)f16(b + 2) * mn[u];
        return;
    }
    case T_Q6_K: *wscale = (double)f16(b + 208) * (double)(int8_t)b[192 + u]; *offs = 0.0; return;
    case T_TQ2_0: *wscale = f16(b + 64); *offs = f16(b + 64); return;
    case T_IQ2_XXS: {
        const uint32_t aux1 = rd32(b + 2 + 8 * u + 4);
        *wscale = (double)f16(b) * (0.125 + 0.25 * (double)(aux1 >> 28));
        *offs = 0.0;
        return;
    }
    case T_MXFP4: *wscale = mxfp4_scale(b[0]); *offs = 0.0; return;
    case T_IQ3_S: *wscale = (double)f16(b) * (double)(1 + 2 * iq3s_scale(b, u)); *offs = 0.0; return;
    case T_IQ3_XXS: *wscale = (double)f16(b) * (0.25 + 0.5 * (double)(rd32(b + 66 + 4 * u) >> 28)); *offs = 0.0; return;
    case T_IQ4_XS: {
        const int sh = b[2] | (b[3] << 8);
        const int ls = ((b[4 + u / 2] >> (4 * (u & 1))) & 15) | (((sh >> (2 * u)) & 3) << 4);
        *wscale = (double)f16(b) * (double)(ls - 32);
        *offs = 0.0;
        return;
    }
    }
    *wscale = *offs = 0.0;
}

/*
 * y[t][r] (fp64) of the integer path for n_tok tokens, from exact int32 sums:
 *   sum over units u of  wscale_u * xd_g * (S_u + S2_u / 254) - offs_u * xs_g   (g: 32-value group of u;
 *   the offset term is applied once per 32-value group)
 * n_threads > 0 parallelises over rows with OpenMP.
 */
int orc_mv(int fmt, const uint8_t* w, int n_out, int n_in, const int8_t* xq, const int8_t* xq2,
           const float* xd, const float* xs, int n_tok, double* y, int n_threads) {
    const int bv = orc_block_values(fmt), bb = orc_block_bytes(fmt), uv = orc_unit_values(fmt);
    if (!bv || n_in % bv) return 2;
    const long long row_bytes = (long long)(n_in / bv) * bb;
    const int upb = bv / uv;   /* units per block */
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(static) if (n_threads > 1)
#endif
    for (int r = 0; r < n_out; ++r) {
        for (int t = 0; t < n_tok; ++t) {
            const int8_t* q = xq + (long long)t * n_in;
            const int8_t* q2 = xq2 + (long long)t * n_in;
            const float* dd = xd + (long long)t * (n_in / 32);
            const float* ss = xs + (long long)t * (n_in / 32);
            double acc = 0.0;
            for (int blk = 0; blk < n_in / bv; ++blk) {
                const uint8_t* b = w + r * row_bytes + (long long)blk * bb;
                for (int ub = 0; ub < upb; ++ub) {
                    int32_t a = 0, a2 = 0, qa = 0, qa2 = 0;
                    const int v0 = blk * bv + ub * uv;
                    for (int i = 0; i < uv; ++i) {
                        const int c = code_of(fmt, b, ub * uv + i);
                        a += c * q[v0 + i];
                        a2 += c * q2[v0 + i];
                        qa += q[v0 + i];
                        qa2 += q2[v0 + i];
                    }
                    double wscale, offs;
                    unit_scales(fmt, b, ub, &wscale, &offs);
                    const int g = v0 / 32;
                    acc += wscale * (double)dd[g] * ((double)a + (double)a2 / 254.0);
                    if (fmt == T_Q2_K) acc -= offs * (double)dd[g] * ((double)qa + (double)qa2 / 254.0);
                    else if (v0 % 32 == 0) acc -= offs * (double)ss[g];
                }
            }
            y[(long long)t * n_out + r] = acc;
        }
    }
    return 0;
}

int orc_version(void) { return 1; }
