"""Seeded synthetic GGUF weights and activations with the value distributions of the benchmark configs.

The reference names no dataset or public benchmark for this path; its configs are synthetic.  The
generators below follow each config's stated distributions and write the exact GGUF block layouts
(ggufengine/quant.py documents them: Q4_0 :60, Q4_1 :67, Q5_0 :83, Q5_1 :90, IQ4_NL :264, Q1_0 :424,
Q2_0 :410, Q2_K :284, Q3_K :295, TQ1_0 :449, IQ2_XS :310, IQ2_S :248, Q8_0 :46, Q4_K :111, Q5_K :123, Q6_K :140, IQ3_XXS :322, IQ3_S :334, IQ4_XS :378, MXFP4 :394, TQ2_0 :417,
IQ2_XXS :235).  Everything is torch, so it runs on the CPU (tests) or on the GPU (bench, where the
largest stacks are several GB).
"""
from __future__ import annotations

from typing import Optional

import torch

from .formats import FORMATS, row_bytes


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=torch.device(device))
    g.manual_seed(seed)
    return g


def _f16_bytes(v: torch.Tensor) -> torch.Tensor:
    """(nb,) float -> (nb, 2) uint8 little-endian fp16."""
    return v.to(torch.float16).contiguous().view(torch.uint8).view(-1, 2)


def _abs_normal(nb: int, scale: float, g, device) -> torch.Tensor:
    return torch.randn(nb, generator=g, device=device).abs() * scale


def _bytes(nb: int, width: int, g, device) -> torch.Tensor:
    return torch.randint(0, 256, (nb, width), generator=g, device=device, dtype=torch.uint8)


def pack_scale_min_k4(sc: torch.Tensor, mn: torch.Tensor) -> torch.Tensor:
    """Inverse of the Q4_K 6-bit scale/min unpacking (ggufengine/quant.py:99-108):
    sc, mn (nb, 8) in 0..63 -> (nb, 12) uint8."""
    sc = sc.to(torch.int32)
    mn = mn.to(torch.int32)
    out = torch.empty(sc.shape[0], 12, dtype=torch.int32, device=sc.device)
    out[:, 0:4] = (sc[:, 0:4] & 63) | ((sc[:, 4:8] >> 4) << 6)
    out[:, 4:8] = (mn[:, 0:4] & 63) | ((mn[:, 4:8] >> 4) << 6)
    out[:, 8:12] = (sc[:, 4:8] & 15) | ((mn[:, 4:8] & 15) << 4)
    return out.to(torch.uint8)


def blocks(fmt: str, n_rows: int, n_in: int, seed: int = 0, device="cpu",
           generator: Optional[torch.Generator] = None) -> torch.Tensor:
    """Random GGUF blocks for an (n_rows, n_in) matrix -> flat uint8 tensor (n_rows * row_bytes)."""
    bv, bb = FORMATS[fmt]
    if n_in % bv:
        raise ValueError(f"{fmt}: n_in {n_in} is not a multiple of {bv}")
    device = torch.device(device)
    g = generator if generator is not None else _gen(seed, device)
    nb = n_rows * n_in // bv
    if fmt == "Q4_0":                       # d = |N(0,1)| * 0.01, nibbles uniform 0..15
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.01, g, device)), _bytes(nb, 16, g, device)], 1)
    elif fmt == "Q4_1":                     # d = |N| * 0.01, m = -|N| * 0.08, nibbles uniform
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.01, g, device)), _f16_bytes(-_abs_normal(nb, 0.08, g, device)),
                         _bytes(nb, 16, g, device)], 1)
    elif fmt == "Q5_0":                     # d = |N| * 0.005; qh and nibbles uniform
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.005, g, device)), _bytes(nb, 20, g, device)], 1)
    elif fmt == "Q5_1":                     # d = |N| * 0.005, m = -|N| * 0.08; qh and nibbles uniform
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.005, g, device)), _f16_bytes(-_abs_normal(nb, 0.08, g, device)),
                         _bytes(nb, 20, g, device)], 1)
    elif fmt == "IQ4_NL":                   # d = |N| * 0.01 / 127; codebook indices uniform
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.01 / 127, g, device)), _bytes(nb, 16, g, device)], 1)
    elif fmt in ("IQ2_XS", "IQ2_S"):        # d = |N| * 0.01; indices, signs, scales uniform
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.01, g, device)), _bytes(nb, bb - 2, g, device)], 1)
    elif fmt == "TQ1_0":                    # trit bytes uniform; d = |N| * 0.01
        out = torch.cat([_bytes(nb, 52, g, device), _f16_bytes(_abs_normal(nb, 0.01, g, device))], 1)
    elif fmt == "Q2_K":                     # scale/min bytes and codes uniform; d, dmin = |N| * 0.005
        out = torch.cat([_bytes(nb, 80, g, device), _f16_bytes(_abs_normal(nb, 0.005, g, device)),
                         _f16_bytes(_abs_normal(nb, 0.005, g, device))], 1)
    elif fmt == "Q3_K":                     # hmask, qs, 6-bit scales uniform; d = |N| * 0.005 / 8
        out = torch.cat([_bytes(nb, 108, g, device), _f16_bytes(_abs_normal(nb, 0.005 / 8, g, device))], 1)
    elif fmt in ("Q1_0", "Q2_0", "PQ2_0"):  # d = |N| * 0.01; code bits uniform
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.01, g, device)), _bytes(nb, bb - 2, g, device)], 1)
    elif fmt == "Q8_0":                     # d = |N| * 0.002, q uniform -127..127
        q = torch.randint(-127, 128, (nb, 32), generator=g, device=device, dtype=torch.int16).to(torch.int8)
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.002, g, device)), q.view(torch.uint8)], 1)
    elif fmt == "Q4_K":                     # d, dmin = |N| * 0.005; 6-bit sc/m uniform; nibbles uniform
        d = _f16_bytes(_abs_normal(nb, 0.005, g, device))
        dmin = _f16_bytes(_abs_normal(nb, 0.005, g, device))
        sc = torch.randint(0, 64, (nb, 8), generator=g, device=device, dtype=torch.int32)
        mn = torch.randint(0, 64, (nb, 8), generator=g, device=device, dtype=torch.int32)
        out = torch.cat([d, dmin, pack_scale_min_k4(sc, mn), _bytes(nb, 128, g, device)], 1)
    elif fmt == "Q5_K":                     # as Q4_K, plus the fifth bits qh[32] uniform
        d = _f16_bytes(_abs_normal(nb, 0.005, g, device))
        dmin = _f16_bytes(_abs_normal(nb, 0.005, g, device))
        sc = torch.randint(0, 64, (nb, 8), generator=g, device=device, dtype=torch.int32)
        mn = torch.randint(0, 64, (nb, 8), generator=g, device=device, dtype=torch.int32)
        out = torch.cat([d, dmin, pack_scale_min_k4(sc, mn), _bytes(nb, 160, g, device)], 1)
    elif fmt == "Q6_K":                     # ql/qh uniform; int8 scales uniform -32..31; d = |N| * 0.005
        ql = _bytes(nb, 192, g, device)
        sc = torch.randint(-32, 32, (nb, 16), generator=g, device=device, dtype=torch.int16).to(torch.int8)
        out = torch.cat([ql, sc.view(torch.uint8), _f16_bytes(_abs_normal(nb, 0.005, g, device))], 1)
    elif fmt == "TQ2_0":                    # ternary codes 0/1/2 (value -1/0/+1) with p = 0.3/0.4/0.3
        u = torch.rand(nb, 2, 4, 32, generator=g, device=device)
        code = (u >= 0.3).to(torch.int32) + (u >= 0.7).to(torch.int32)
        shifts = (2 * torch.arange(4, device=device, dtype=torch.int32)).view(1, 1, 4, 1)
        qs = (code << shifts).sum(2).to(torch.uint8).view(nb, 64)      # byte 32n+m: value 128n+32g+m at bits 2g
        out = torch.cat([qs, _f16_bytes(_abs_normal(nb, 0.01, g, device))], 1)
    elif fmt == "IQ2_XXS":                  # d = |N| * 0.01; grid index, sign index, 4-bit scale uniform
        d = _f16_bytes(_abs_normal(nb, 0.01, g, device))
        grid = _bytes(nb * 8, 4, g, device)
        sign = torch.randint(0, 128, (nb * 8, 4), generator=g, device=device, dtype=torch.int64)
        scale = torch.randint(0, 16, (nb * 8,), generator=g, device=device, dtype=torch.int64)
        aux1 = (sign[:, 0] | (sign[:, 1] << 7) | (sign[:, 2] << 14) | (sign[:, 3] << 21) | (scale << 28))
        aux1 = aux1 - ((aux1 >> 31) << 32)                                        # as signed 32-bit
        aux1 = aux1.to(torch.int32).contiguous().view(torch.uint8).view(nb * 8, 4)   # little endian
        out = torch.cat([d, torch.cat([grid, aux1], 1).view(nb, 64)], 1)
    elif fmt == "IQ4_XS":                   # d = |N| * 0.01 / 32; 6-bit sub-block scales and nibbles uniform
        d = _f16_bytes(_abs_normal(nb, 0.01 / 32, g, device))
        out = torch.cat([d, _bytes(nb, 134, g, device)], 1)
    elif fmt == "IQ3_XXS":                  # d = |N| * 0.01 / 32; grid indices, sign groups, scales uniform
        d = _f16_bytes(_abs_normal(nb, 0.01 / 32, g, device))
        out = torch.cat([d, _bytes(nb, 96, g, device)], 1)
    elif fmt == "IQ3_S":                    # d = |N| * 0.01 / 16; grid indices, signs and 4-bit scales uniform
        d = _f16_bytes(_abs_normal(nb, 0.01 / 16, g, device))
        out = torch.cat([d, _bytes(nb, 108, g, device)], 1)
    elif fmt == "IQ1_S":                    # d = |N| * 0.01 / 8; grid indices, 3-bit scales, delta signs uniform
        out = torch.cat([_f16_bytes(_abs_normal(nb, 0.01 / 8, g, device)), _bytes(nb, 48, g, device)], 1)
    elif fmt == "IQ1_M":                    # index bytes and nibbles, 3-bit scales uniform; d = |N| * 0.01 / 8 in
        body = _bytes(nb, 48, g, device)     # the top nibbles of the four scale words
        sc = torch.randint(0, 4096, (nb, 4), generator=g, device=device, dtype=torch.int32)
        d = _abs_normal(nb, 0.01 / 8, g, device).to(torch.float16).view(torch.int16).to(torch.int32) & 0xFFFF
        sc = sc | (((d.view(nb, 1) >> (4 * torch.arange(4, device=device, dtype=torch.int32))) & 0xF) << 12)
        sc = (sc - ((sc >> 15) << 16)).to(torch.int16).contiguous().view(torch.uint8).view(nb, 8)
        out = torch.cat([body, sc], 1)
    elif fmt == "PTQ1_0":                   # trit bytes uniform; d = |N| * 0.01
        out = torch.cat([_bytes(nb, 26, g, device), _f16_bytes(_abs_normal(nb, 0.01, g, device))], 1)
    elif fmt == "MXFP4":                    # scale 2^(e-128) with e uniform 118..124; nibbles uniform
        e = torch.randint(118, 125, (nb, 1), generator=g, device=device, dtype=torch.int32).to(torch.uint8)
        out = torch.cat([e, _bytes(nb, 16, g, device)], 1)
    else:
        raise ValueError(f"unsupported format {fmt}")
    assert out.shape[1] == bb
    return out.reshape(-1).contiguous()


def activations(n_tok: int, n_in: int, seed: int = 0, device="cpu", dtype=torch.float32) -> torch.Tensor:
    """x ~ N(0, 1), shape (n_tok, n_in)."""
    g = _gen(seed, device)
    return torch.randn(n_tok, n_in, generator=g, device=device).to(dtype)


def router_logits(n_tok: int, n_exp: int, seed: int = 0, device="cpu") -> torch.Tensor:
    g = _gen(seed, device)
    return torch.randn(n_tok, n_exp, generator=g, device=device)


def matrix_bytes(fmt: str, n_rows: int, n_in: int) -> int:
    return n_rows * row_bytes(fmt, n_in)
