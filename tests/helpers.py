"""Shared test data: seeded GGUF blocks (synthetic configs) and their oracle results."""
from __future__ import annotations

import numpy as np
import torch

from nemicli_terminal_b200 import synth
from nemicli_terminal_b200.formats import FORMATS
from oracle import oracle as O

FMTS = tuple(FORMATS)


def case(fmt: str, n_out: int, n_in: int, n_tok: int = 1, seed: int = 0, x_dtype=torch.float32):
    """(raw uint8 CPU tensor, x CPU tensor (n_tok, n_in))."""
    raw = synth.blocks(fmt, n_out, n_in, seed=seed)
    x = synth.activations(n_tok, n_in, seed=seed + 1000).to(x_dtype)
    return raw, x


def x_numpy(x: torch.Tensor) -> np.ndarray:
    """The activation as the oracle takes it: fp32, or uint16 bf16 bits."""
    if x.dtype == torch.float32:
        return x.contiguous().numpy()
    if x.dtype == torch.bfloat16:
        return x.contiguous().view(torch.int16).numpy().view(np.uint16)
    raise TypeError(x.dtype)


def oracle_b(fmt, raw: torch.Tensor, x: torch.Tensor, n_out: int, n_in: int):
    """Integer-path oracle: (y fp64 (T, n_out), (xq, xq2, xd, xs))."""
    T = x.shape[0]
    qa = O.quant_q8(x_numpy(x).reshape(-1))
    y = O.mv(fmt, raw.numpy(), n_out, n_in, *qa, n_tok=T)
    return y, qa


def oracle_a(fmt, raw: torch.Tensor, x: torch.Tensor, n_out: int, n_in: int) -> np.ndarray:
    """Dequantise-and-matmul oracle with the unquantised activation (fp64)."""
    xf = x.float().numpy()
    return O.mv_exact(fmt, raw.numpy(), n_out, n_in, xf)
