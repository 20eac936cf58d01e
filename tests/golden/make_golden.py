"""Generates tests/golden/dequant_golden.npz from the reference engine's own dequantiser.

Run once where the reference checkout is available (it does not travel to the GPU box):

    python tests/golden/make_golden.py <reference root>

For each in-scope format it stores seeded raw GGUF blocks, the reference's
ggufengine.quant.dequantize output for them (fp32), a seeded fp32 activation and the fp64 product
dequant @ x.  Scale fields are set to small finite fp16 values (the pattern of the reference's
tests/test_gguf_iq.py:81-101, zufallsbloecke).  Extra cases pin the corners:

* IQ2_XXS blocks whose grid indices run through all 256 codebook entries and whose sign indices
  run through all 128 patterns,
* TQ2_0 blocks with every 2-bit code, including the never-drawn code 3,
* Q4_K blocks with 6-bit scales and mins at 0 and 63,
* Q5_K blocks with scales and mins at 0 and 63 and every fifth bit (qh) set or clear,
* IQ4_XS blocks whose sub-block scales run through all 64 values and whose nibbles run through all 16
  codebook entries,
* MXFP4 blocks with every nibble and scale exponents from the subnormal range (0, 1) up to 200,
* IQ3_S blocks whose grid indices run through all 512 codebook entries, whose sign bytes run through
  all 256 patterns and whose scales run through all 16 values,
* IQ3_XXS blocks whose grid indices run through all 256 codebook entries, whose sign groups run through
  all 128 patterns and whose scales run through all 16 values,
* Q5_0 / Q5_1 blocks with every fifth bit set and with every fifth bit clear,
* Q2_0 / PQ2_0 blocks with every 2-bit code (3, never written by the quantiser, included),
* Q3_K blocks with every 6-bit scale (-32..31) and every high bit set or clear,
* IQ2_XS / IQ2_S blocks whose codebook indices run through all 512 / 1024 entries, with every sign
  pattern and every 4-bit scale,
* Q2_K blocks with every scale/min byte,
* TQ1_0 blocks with every byte value in every trit position,
* IQ1_S / IQ1_M blocks whose grid indices run through all 2048 codebook entries, with every 3-bit scale
  and both delta signs,
* PTQ1_0 blocks with every byte value in every qs and qh position.

Formats added later are generated after the earlier cases, so the earlier arrays stay as they were.
"""
from __future__ import annotations

import os
import sys

import numpy as np

FORMATS = {"Q4_0": (2, 32, 18), "Q8_0": (8, 32, 34), "Q4_K": (12, 256, 144), "Q6_K": (14, 256, 210),
           "IQ2_XXS": (16, 256, 66), "TQ2_0": (35, 256, 66)}
LATER = {"Q5_K": (13, 256, 176)}
LATER2 = {"IQ4_XS": (23, 256, 136)}
LATER3 = {"MXFP4": (39, 32, 17)}
LATER4 = {"IQ3_S": (21, 256, 110)}
LATER5 = {"IQ3_XXS": (18, 256, 98)}
LATER6 = {"Q4_1": (3, 32, 20), "Q5_0": (6, 32, 22), "Q5_1": (7, 32, 24), "IQ4_NL": (20, 32, 18)}
LATER7 = {"Q1_0": (41, 128, 18), "Q2_0": (42, 64, 18), "PQ2_0": (142, 128, 34)}
LATER8 = {"Q3_K": (11, 256, 110)}
LATER9 = {"IQ2_XS": (17, 256, 74), "IQ2_S": (22, 256, 82)}
LATER10 = {"Q2_K": (10, 256, 84)}
LATER11 = {"TQ1_0": (34, 256, 54)}
LATER12 = {"IQ1_S": (19, 256, 50), "IQ1_M": (29, 256, 56), "PTQ1_0": (143, 128, 28)}
SCALE_OFFSETS = {"Q4_0": (0,), "Q8_0": (0,), "Q4_K": (0, 2), "Q6_K": (208,), "IQ2_XXS": (0,), "TQ2_0": (64,),
                 "Q5_K": (0, 2), "IQ4_XS": (0,), "MXFP4": (), "IQ3_S": (0,), "IQ3_XXS": (0,),
                 "Q4_1": (0, 2), "Q5_0": (0,), "Q5_1": (0, 2), "IQ4_NL": (0,), "Q1_0": (0,), "Q2_0": (0,),
                 "PQ2_0": (0,), "Q3_K": (108,), "IQ2_XS": (0,), "IQ2_S": (0,), "Q2_K": (80, 82), "TQ1_0": (52,),
                 "IQ1_S": (0,), "IQ1_M": (), "PTQ1_0": (26,)}
ROWS, COLS = 3, 512          # a (3, 512) matrix per format


def random_blocks(name: str, n_blocks: int, rng: np.random.Generator) -> np.ndarray:
    _, _, size = {**FORMATS, **LATER, **LATER2, **LATER3, **LATER4, **LATER5, **LATER6, **LATER7, **LATER8,
                  **LATER9, **LATER10, **LATER11, **LATER12}[name]
    raw = rng.integers(0, 256, (n_blocks, size), dtype=np.uint8)
    if name == "IQ1_M":                                 # d's four nibbles in the top bits of the scale words
        d = (rng.random(n_blocks) * 0.01 + 0.001).astype(np.float16).view(np.uint16).astype(np.uint32)
        sc = raw[:, 48:56].copy().view(np.uint16).astype(np.uint32) & 0x0FFF
        for i in range(4):
            sc[:, i] |= ((d >> (4 * i)) & 0xF) << 12
        raw[:, 48:56] = sc.astype(np.uint16).view(np.uint8).reshape(n_blocks, 8)
    if name == "MXFP4":
        raw[:, 0] = rng.integers(118, 125, n_blocks)       # scale exponents 2^-10 .. 2^-4
    for o in SCALE_OFFSETS[name]:
        d = (rng.random(n_blocks) * 0.01 + 0.001).astype(np.float16)
        raw[:, o:o + 2] = d.view(np.uint8).reshape(n_blocks, 2)
    return raw


def iq2xxs_cover(rng: np.random.Generator) -> np.ndarray:
    """8 blocks = 64 sub-blocks = 256 grid slots: grid index k at slot k; sign index k % 128."""
    raw = random_blocks("IQ2_XXS", 8, rng)
    for sb in range(64):
        blk, ib = divmod(sb, 8)
        o = 2 + 8 * ib
        idx = [4 * sb + l for l in range(4)]
        raw[blk, o:o + 4] = np.array(idx, dtype=np.uint8)
        signs = [(4 * sb + l) % 128 for l in range(4)]
        aux1 = signs[0] | (signs[1] << 7) | (signs[2] << 14) | (signs[3] << 21) | ((sb % 16) << 28)
        raw[blk, o + 4:o + 8] = np.frombuffer(np.uint32(aux1).tobytes(), dtype=np.uint8)
    return raw


def tq2_cover(rng: np.random.Generator) -> np.ndarray:
    raw = random_blocks("TQ2_0", 2, rng)
    raw[:, :64] = np.arange(128, dtype=np.uint8).reshape(2, 64) * 2 + 1    # mixes all 2-bit codes
    raw[0, :4] = 0xFF                                                       # code 3 everywhere
    return raw


def q4k_cover(rng: np.random.Generator) -> np.ndarray:
    raw = random_blocks("Q4_K", 2, rng)
    raw[0, 4:16] = 0xFF        # every 6-bit scale and min = 63
    raw[1, 4:16] = 0x00        # every 6-bit scale and min = 0
    return raw


def q5k_cover(rng: np.random.Generator) -> np.ndarray:
    raw = random_blocks("Q5_K", 2, rng)
    raw[0, 4:16] = 0xFF        # every 6-bit scale and min = 63
    raw[0, 16:48] = 0xFF       # every fifth bit set: codes 16..31
    raw[1, 4:16] = 0x00        # every 6-bit scale and min = 0
    raw[1, 16:48] = 0x00       # every fifth bit clear
    return raw


def iq4xs_cover(rng: np.random.Generator) -> np.ndarray:
    """8 blocks = 64 sub-blocks: sub-block k has 6-bit scale k; byte j of a sub-block holds nibbles
    j and 15 - j."""
    raw = random_blocks("IQ4_XS", 8, rng)
    for blk in range(8):
        sh, sl = 0, [0, 0, 0, 0]
        for ib in range(8):
            ls = 8 * blk + ib
            sl[ib // 2] |= (ls & 15) << (4 * (ib & 1))
            sh |= (ls >> 4) << (2 * ib)
            raw[blk, 8 + 16 * ib:8 + 16 * ib + 16] = [j | ((15 - j) << 4) for j in range(16)]
        raw[blk, 2:4] = [sh & 0xFF, sh >> 8]
        raw[blk, 4:8] = sl
    return raw


def mxfp4_cover(rng: np.random.Generator) -> np.ndarray:
    """16 blocks: byte j of every block holds nibbles j and 15 - j; exponents 0..3, 100, 126..130, 200."""
    raw = random_blocks("MXFP4", 16, rng)
    raw[:, 0] = [0, 1, 2, 3, 100, 126, 127, 128, 129, 130, 200, 120, 121, 122, 123, 124]
    raw[:, 1:17] = [j | ((15 - j) << 4) for j in range(16)]
    return raw


def iq3s_cover(rng: np.random.Generator) -> np.ndarray:
    """8 blocks = 512 grid slots: grid index k at slot k; sign byte k % 256; scale k % 16 per sub-block."""
    raw = random_blocks("IQ3_S", 8, rng)
    for blk in range(8):
        idx = [64 * blk + g for g in range(64)]
        raw[blk, 2:66] = [i & 0xFF for i in idx]
        raw[blk, 66:74] = [sum(((idx[8 * i + j] >> 8) & 1) << j for j in range(8)) for i in range(8)]
        raw[blk, 74:106] = [(32 * blk + j) % 256 for j in range(32)]
        raw[blk, 106:110] = [((8 * blk + 2 * i) % 16) | (((8 * blk + 2 * i + 1) % 16) << 4) for i in range(4)]
    return raw


def iq3xxs_cover(rng: np.random.Generator) -> np.ndarray:
    """4 blocks = 256 grid slots: grid index k at slot k; sign group k % 128; scale per sub-block."""
    raw = random_blocks("IQ3_XXS", 4, rng)
    for blk in range(4):
        raw[blk, 2:66] = [64 * blk + k for k in range(64)]
        for ib in range(8):
            signs = [(32 * blk + 4 * ib + l) % 128 for l in range(4)]
            aux = signs[0] | (signs[1] << 7) | (signs[2] << 14) | (signs[3] << 21) | (((8 * blk + ib) % 16) << 28)
            raw[blk, 66 + 4 * ib:70 + 4 * ib] = np.frombuffer(np.uint32(aux).tobytes(), dtype=np.uint8)
    return raw


def q5_cover(name: str, rng: np.random.Generator) -> np.ndarray:
    raw = random_blocks(name, 16, rng)
    o = 4 if name == "Q5_1" else 2
    raw[:8, o:o + 4] = 0xFF
    raw[8:, o:o + 4] = 0x00
    return raw


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    import torch
    from ggufengine.quant import dequantize      # the reference's dequantiser (ggufengine/quant.py:484)

    rng = np.random.default_rng(20260101)
    out = {}

    def add(key: str, name: str, raw: np.ndarray, rows: int, cols: int) -> None:
        t, bv, bb = {**FORMATS, **LATER, **LATER2, **LATER3, **LATER4, **LATER5, **LATER6, **LATER7, **LATER8,
                     **LATER9, **LATER10, **LATER11, **LATER12}[name]
        flat = np.ascontiguousarray(raw.reshape(-1))
        assert flat.size == rows * cols // bv * bb
        deq = dequantize(torch.from_numpy(flat.copy()), t, rows * cols, torch.float32).numpy()
        x = rng.standard_normal((2, cols)).astype(np.float32)
        y = x.astype(np.float64) @ deq.reshape(rows, cols).astype(np.float64).T
        out[f"{key}__raw"] = flat
        out[f"{key}__deq"] = deq.astype(np.float32)
        out[f"{key}__x"] = x
        out[f"{key}__y"] = y
        out[f"{key}__shape"] = np.array([t, rows, cols], dtype=np.int64)

    for name, (_, bv, _) in FORMATS.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    add("IQ2_XXS_cover", "IQ2_XXS", iq2xxs_cover(rng), 8, 256)
    add("TQ2_0_cover", "TQ2_0", tq2_cover(rng), 2, 256)
    add("Q4_K_cover", "Q4_K", q4k_cover(rng), 2, 256)
    for name, (_, bv, _) in LATER.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    add("Q5_K_cover", "Q5_K", q5k_cover(rng), 2, 256)
    for name, (_, bv, _) in LATER2.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    add("IQ4_XS_cover", "IQ4_XS", iq4xs_cover(rng), 8, 256)
    for name, (_, bv, _) in LATER3.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    add("MXFP4_cover", "MXFP4", mxfp4_cover(rng), 2, 256)
    for name, (_, bv, _) in LATER4.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    add("IQ3_S_cover", "IQ3_S", iq3s_cover(rng), 8, 256)
    for name, (_, bv, _) in LATER5.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    add("IQ3_XXS_cover", "IQ3_XXS", iq3xxs_cover(rng), 4, 256)
    for name, (_, bv, _) in LATER6.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    add("Q5_0_cover", "Q5_0", q5_cover("Q5_0", rng), 2, 256)
    add("Q5_1_cover", "Q5_1", q5_cover("Q5_1", rng), 2, 256)
    for name, (_, bv, _) in LATER7.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    for name, per in (("Q2_0", 4), ("PQ2_0", 2)):
        raw = random_blocks(name, per, rng)
        raw[:, 2:] = np.arange(raw[:, 2:].size, dtype=np.uint32).reshape(raw[:, 2:].shape) % 256
        add(name + "_cover", name, raw, 1, 256)
    for name, (_, bv, _) in LATER8.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    raw = random_blocks("Q3_K", 4, rng)                      # 64 scale groups: every 6-bit scale once
    for blk in range(4):
        sc = [16 * blk + i for i in range(16)]
        raw[blk, 96:104] = [(sc[i] & 15) | ((sc[i + 8] & 15) << 4) for i in range(8)]
        raw[blk, 104:108] = [sum(((sc[4 * s + i] >> 4) & 3) << (2 * s) for s in range(4)) for i in range(4)]
    raw[0, :32] = 0xFF
    raw[1, :32] = 0x00
    add("Q3_K_cover", "Q3_K", raw, 4, 256)
    for name, (_, bv, _) in LATER9.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    raw = random_blocks("IQ2_XS", 16, rng)                   # 512 entries: index k, sign index k % 128
    for blk in range(16):
        for e in range(32):
            k = 32 * blk + e
            q = (k & 511) | ((k % 128) << 9)
            raw[blk, 2 + 2 * e:4 + 2 * e] = [q & 0xFF, q >> 8]
        raw[blk, 66:74] = [(blk + 2 * i) % 16 | (((blk + 2 * i + 1) % 16) << 4) for i in range(8)]
    add("IQ2_XS_cover", "IQ2_XS", raw, 16, 256)
    raw = random_blocks("IQ2_S", 32, rng)                    # 1024 entries: index k, sign byte k % 256
    for blk in range(32):
        idx = [32 * blk + e for e in range(32)]
        raw[blk, 2:34] = [i & 0xFF for i in idx]
        raw[blk, 34:66] = [i % 256 for i in idx]
        raw[blk, 66:74] = [sum(((idx[4 * g + j] >> 8) & 3) << (2 * j) for j in range(4)) for g in range(8)]
        raw[blk, 74:82] = [(blk + 2 * i) % 16 | (((blk + 2 * i + 1) % 16) << 4) for i in range(8)]
    add("IQ2_S_cover", "IQ2_S", raw, 32, 256)
    for name, (_, bv, _) in LATER10.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    raw = random_blocks("Q2_K", 16, rng)                     # every scale/min byte once
    raw[:, :16] = np.arange(256, dtype=np.uint8).reshape(16, 16)
    add("Q2_K_cover", "Q2_K", raw, 16, 256)
    for name, (_, bv, _) in LATER11.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    raw = random_blocks("TQ1_0", 6, rng)                     # every byte value in qs and in qh positions
    vals = np.arange(6 * 52, dtype=np.uint32) % 256
    raw[:, :52] = vals.reshape(6, 52)
    add("TQ1_0_cover", "TQ1_0", raw, 6, 256)
    for name, (_, bv, _) in LATER12.items():
        add(name, name, random_blocks(name, ROWS * COLS // bv, rng), ROWS, COLS)
    raw = random_blocks("IQ1_S", 64, rng)          # entry k at slot k; sub-block j: scale j % 8, sign (j // 8) % 2
    for blk in range(64):
        for ib in range(8):
            idx = [32 * blk + 4 * ib + l for l in range(4)]
            raw[blk, 2 + 4 * ib:6 + 4 * ib] = [i & 0xFF for i in idx]
            j = 8 * blk + ib
            qh = sum((i >> 8) << (3 * l) for l, i in enumerate(idx)) | ((j % 8) << 12) | (((j // 8) % 2) << 15)
            raw[blk, 34 + 2 * ib:36 + 2 * ib] = [qh & 0xFF, qh >> 8]
    add("IQ1_S_cover", "IQ1_S", raw, 64, 256)
    raw = random_blocks("IQ1_M", 64, rng)          # entry k at slot k, delta sign k % 2, group scale (blk + g) % 8
    for blk in range(64):
        idx = [32 * blk + e for e in range(32)]
        raw[blk, :32] = [i & 0xFF for i in idx]
        nib = [(i >> 8) | ((e % 2) << 3) for e, i in enumerate(idx)]
        raw[blk, 32:48] = [nib[2 * i] | (nib[2 * i + 1] << 4) for i in range(16)]
        sc = raw[blk, 48:56].copy().view(np.uint16).astype(np.uint32) & 0xF000
        for g in range(16):
            sc[g // 4] |= ((blk + g) % 8) << (3 * (g % 4))
        raw[blk, 48:56] = sc.astype(np.uint16).view(np.uint8)
    add("IQ1_M_cover", "IQ1_M", raw, 64, 256)
    raw = random_blocks("PTQ1_0", 128, rng)        # qs: byte values cycling through 0..255; qh: every value
    raw[:, :24] = (np.arange(128 * 24, dtype=np.uint32) % 256).reshape(128, 24)
    raw[:, 24:26] = np.arange(256, dtype=np.uint32).reshape(128, 2)
    add("PTQ1_0_cover", "PTQ1_0", raw, 16, 1024)
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dequant_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("NEMICLI_REFERENCE", ""))
