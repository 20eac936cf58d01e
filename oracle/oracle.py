"""TEST INFRASTRUCTURE ONLY: Python view of the CPU oracle (qmv_oracle.c) plus numpy helpers.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs only — never by the
product package.  Two oracles live here:

* oracle A, `mv_exact`: dequantise the GGUF blocks (a restatement of ggufengine/quant.py, bit-identical,
  pinned by tests/golden) and multiply with the unquantised fp32 activation in fp64.  This is the
  reference's own dequantise-and-matmul; the north-star bound is 1e-3 max-abs / max-ref against it.
* oracle B, `quant_q8` + `block_sums` + `mv`: the reference's two-stage int8 integer path
  (ggufengine/mmvq.py:59-83 and :341-482), with exact int32 sums per unit and an fp64 epilogue.
  The GPU kernels must reproduce the int32 sums bit for bit from the same activation input.
* oracle C, `mmq`: the reference's tensor-core path for several tokens (ggufengine/mmvq.py:536-724):
  weight values unpacked to fp16 by its fp32 formulas, tokens scaled per row to |x| <= 256 in fp16,
  products summed exactly (fp64) and scaled back.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqmv_oracle.so")

# GGML type ids (ggufengine/gguf.py:64-77) of the twenty-six in-scope formats
TYPES = {"Q4_0": 2, "Q8_0": 8, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14, "IQ2_XXS": 16, "IQ4_XS": 23, "TQ2_0": 35, "MXFP4": 39, "IQ3_S": 21, "IQ3_XXS": 18,
         "Q4_1": 3, "Q5_0": 6, "Q5_1": 7, "IQ4_NL": 20, "Q1_0": 41, "Q2_0": 42, "PQ2_0": 142,
         "Q3_K": 11, "IQ2_XS": 17, "IQ2_S": 22, "Q2_K": 10, "TQ1_0": 34, "IQ1_S": 19, "IQ1_M": 29, "PTQ1_0": 143}
BLOCK = {"Q4_0": (32, 18), "Q8_0": (32, 34), "Q4_K": (256, 144), "Q5_K": (256, 176), "Q6_K": (256, 210),
         "IQ2_XXS": (256, 66), "IQ4_XS": (256, 136), "TQ2_0": (256, 66), "MXFP4": (32, 17),
         "IQ3_S": (256, 110), "IQ3_XXS": (256, 98), "Q4_1": (32, 20), "Q5_0": (32, 22), "Q5_1": (32, 24),
         "IQ4_NL": (32, 18), "Q1_0": (128, 18), "Q2_0": (64, 18), "PQ2_0": (128, 34),
         "Q3_K": (256, 110), "IQ2_XS": (256, 74), "IQ2_S": (256, 82),
         "Q2_K": (256, 84), "TQ1_0": (256, 54), "IQ1_S": (256, 50), "IQ1_M": (256, 56), "PTQ1_0": (128, 28)}

_lock = threading.Lock()
_lib = None


def build() -> str:
    """Compile the oracle with its Makefile (gcc on PATH)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(
                    os.path.join(HERE, "qmv_oracle.c")):
                build()
            L = ctypes.CDLL(LIB_PATH)
            P, I, LL = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong
            L.orc_quant_q8.argtypes = [P, I, LL, P, P, P, P]
            L.orc_quant_q8.restype = None
            L.orc_dequant.argtypes = [I, P, LL, P]
            L.orc_block_sums.argtypes = [I, P, I, I, P, P, P, P]
            L.orc_mv.argtypes = [I, P, I, I, P, P, P, P, I, P, I]
            _lib = L
    return _lib


def _p(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"]
    return ctypes.c_void_p(a.ctypes.data)


def fmt_id(fmt) -> int:
    return TYPES[fmt] if isinstance(fmt, str) else int(fmt)


def quant_q8(x: np.ndarray):
    """x: fp32, or uint16 holding bf16 bits; size % 32 == 0 -> (xq, xq2, xd, xs)."""
    x = np.ascontiguousarray(x)
    n = x.size
    assert n % 32 == 0 and x.dtype in (np.float32, np.uint16)
    xq = np.empty(n, np.int8)
    xq2 = np.empty(n, np.int8)
    xd = np.empty(n // 32, np.float32)
    xs = np.empty(n // 32, np.float32)
    lib().orc_quant_q8(_p(x), int(x.dtype == np.float32), n, _p(xq), _p(xq2), _p(xd), _p(xs))
    return xq, xq2, xd, xs


def dequant(fmt, raw: np.ndarray, n_values: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n_values, np.float32)
    rc = lib().orc_dequant(fmt_id(fmt), _p(raw), n_values, _p(out))
    if rc:
        raise ValueError(f"orc_dequant: status {rc}")
    return out


def unit_values(fmt) -> int:
    return 16 if fmt_id(fmt) in (TYPES["Q6_K"], TYPES["Q3_K"], TYPES["IQ2_XS"], TYPES["IQ2_S"], TYPES["Q2_K"],
                                 TYPES["IQ1_M"]) else 32


def block_sums(fmt, w: np.ndarray, n_out: int, n_in: int, xq: np.ndarray, xq2: np.ndarray):
    """Exact int32 sums per (row, unit) for one token -> (s, s2), shape (n_out, n_in / unit)."""
    units = n_in // unit_values(fmt)
    s = np.empty((n_out, units), np.int32)
    s2 = np.empty((n_out, units), np.int32)
    rc = lib().orc_block_sums(fmt_id(fmt), _p(np.ascontiguousarray(w, dtype=np.uint8)), n_out, n_in,
                              _p(np.ascontiguousarray(xq)), _p(np.ascontiguousarray(xq2)), _p(s), _p(s2))
    if rc:
        raise ValueError(f"orc_block_sums: status {rc}")
    return s, s2


def mv(fmt, w: np.ndarray, n_out: int, n_in: int, xq, xq2, xd, xs, n_tok: int = 1, threads: int = 0) -> np.ndarray:
    """Integer-path matvec, fp64 epilogue: -> (n_tok, n_out) float64."""
    y = np.empty((n_tok, n_out), np.float64)
    rc = lib().orc_mv(fmt_id(fmt), _p(np.ascontiguousarray(w, dtype=np.uint8)), n_out, n_in,
                      _p(np.ascontiguousarray(xq)), _p(np.ascontiguousarray(xq2)), _p(np.ascontiguousarray(xd)),
                      _p(np.ascontiguousarray(xs)), n_tok, _p(y), threads)
    if rc:
        raise ValueError(f"orc_mv: status {rc}")
    return y


def mv_exact(fmt, w: np.ndarray, n_out: int, n_in: int, x: np.ndarray) -> np.ndarray:
    """Oracle A: dequantise (bit-identical to quant.dequantize) and multiply with x (T, n_in) in fp64."""
    W = dequant(fmt, w, n_out * n_in).reshape(n_out, n_in).astype(np.float64)
    x = np.asarray(x, np.float64).reshape(-1, n_in)
    return x @ W.T


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (round to nearest even), as torch's .to(torch.bfloat16)."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def max_rel(y, ref) -> float:
    """max |y - ref| / max |ref| (the reference tests' measure, tests/test_gguf_iq.py:215 there)."""
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-300))


def _f32(a) -> np.ndarray:
    return np.asarray(a, np.float64).astype(np.float32)


def mmq_weights(fmt, w: np.ndarray, n_out: int, n_in: int) -> np.ndarray:
    """Oracle C's fp16 weights (n_out, n_in): Q4_K fp16(fma(d sc, q, -dmin m)) (mmvq.py:578-592), Q6_K
    fp16(d sc (q - 32)) (mmvq.py:606-616), each product and difference rounded to fp32 as there."""
    nb = n_in // 256
    if fmt == "Q4_K":
        b = np.asarray(w, np.uint8).reshape(n_out * nb, 144)
        d = b[:, 0:2].copy().view(np.float16).astype(np.float32)[:, 0]
        dm = b[:, 2:4].copy().view(np.float16).astype(np.float32)[:, 0]
        s = b[:, 4:16].astype(np.int32)
        sc = np.empty((len(b), 8), np.int32)
        mn = np.empty((len(b), 8), np.int32)
        for j in range(8):
            if j < 4:
                sc[:, j], mn[:, j] = s[:, j] & 63, s[:, j + 4] & 63
            else:
                sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
                mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
        qs = b[:, 16:144].astype(np.int32).reshape(-1, 4, 32)
        q = np.empty((len(b), 8, 32), np.int32)
        q[:, 0::2] = qs & 15
        q[:, 1::2] = qs >> 4
        a = _f32(d[:, None].astype(np.float64) * sc)                 # d sc, rounded to fp32
        c = _f32(dm[:, None].astype(np.float64) * mn)                # dmin m
        v = _f32(a[:, :, None].astype(np.float64) * q - c[:, :, None])   # one fused multiply-add
        return v.astype(np.float16).reshape(n_out, n_in)
    if fmt == "Q6_K":
        b = np.asarray(w, np.uint8).reshape(n_out * nb, 210)
        ql = b[:, 0:128].astype(np.int32)
        qh = b[:, 128:192].astype(np.int32)
        sc = b[:, 192:208].view(np.int8).astype(np.int32)
        d = b[:, 208:210].copy().view(np.float16).astype(np.float32)[:, 0]
        v = np.empty((len(b), 256), np.float32)
        l = np.arange(32)
        for n in range(2):
            for g, (lo, sh, hi_sh) in enumerate(((0, 0, 0), (32, 0, 2), (0, 4, 4), (32, 4, 6))):
                q = ((ql[:, 64 * n + lo + l] >> sh) & 0xF) | (((qh[:, 32 * n + l] >> hi_sh) & 3) << 4)
                f = _f32(d[:, None].astype(np.float64) * sc[:, 8 * n + l // 16 + 2 * g])
                v[:, 128 * n + 32 * g + l] = _f32(f.astype(np.float64) * (q - 32))
        return v.astype(np.float16).reshape(n_out, n_in)
    raise ValueError(f"mmq: {fmt} (Q4_K, Q6_K)")


def mmq_input(x: np.ndarray):
    """Tokens (T, n) fp32 -> (fp16 values x / xs, xs): xs = max(max|x|, 1e-30) / 256 (mmvq.py:617-640)."""
    x = np.asarray(x, np.float32)
    m = np.abs(x).max(axis=1)
    xs = _f32(np.maximum(m, np.float32(1e-30)).astype(np.float64) / 256.0)
    inv = _f32(1.0 / xs.astype(np.float64))
    xh = _f32(x.astype(np.float64) * inv[:, None]).astype(np.float16)
    return xh, xs


def mmq(fmt, w: np.ndarray, n_out: int, n_in: int, x: np.ndarray) -> np.ndarray:
    """Oracle C: (T, n_in) fp32 tokens -> (T, n_out) fp64, the reference MMQ's values summed exactly."""
    W = mmq_weights(fmt, w, n_out, n_in).astype(np.float64)
    xh, xs = mmq_input(np.asarray(x, np.float32).reshape(-1, n_in))
    return (xh.astype(np.float64) @ W.T) * xs.astype(np.float64)[:, None]
