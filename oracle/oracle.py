"""TEST INFRASTRUCTURE ONLY: Python view of the CPU oracle (qmv_oracle.c) plus numpy helpers.

Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs only — never by the
product package.  Two oracles live here:

* oracle A, `mv_exact`: dequantise the GGUF blocks (a restatement of ggufengine/quant.py, bit-identical,
  pinned by tests/golden) and multiply with the unquantised fp32 activation in fp64.  This is the
  reference's own dequantise-and-matmul; the north-star bound is 1e-3 max-abs / max-ref against it.
* oracle B, `quant_q8` + `block_sums` + `mv`: the reference's two-stage int8 integer path
  (ggufengine/mmvq.py:59-83 and :341-482), with exact int32 sums per unit and an fp64 epilogue.
  The GPU kernels must reproduce the int32 sums bit for bit from the same activation input.
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
