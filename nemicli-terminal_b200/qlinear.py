"""Drop-in for the reference's QuantLinear (ggufengine/qlinear.py:195-276), the GPU route of dense Q4_0
and Q8_0 matrices (and of Q4_K / Q6_K where the reference's int8 kernels are unavailable).

The reference repacks the GGUF blocks at load time into tinygemm's int4 tile layout and runs
torch._weight_int4pack_mm (one call for 4-bit formats, two for 8-bit ones).  This version keeps the
GGUF bytes as they are and runs this package's int8 matvec kernels on them: no repack, no second pass
for Q8_0, and the same bytes can still be shared with an embedding table.  The call signature, output
dtype (bf16) and bias handling are the reference's.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib, mmvq
from .formats import FORMATS, GGML_TYPES

G = 32                                     # group size along K (reference qlinear.py:33)
UNPACK_FROM = 256                          # from this many rows: unpack to bf16 + cuBLAS (reference qlinear.py:36)
_QUANT = ("Q4_0", "Q8_0", "Q4_K", "Q6_K")  # formats this QuantLinear takes


class GGUFError(ValueError):
    pass


def kernel_available(device: torch.device) -> bool:
    """The kernels run on this device (reference qlinear.py:42-43)."""
    from . import _lib
    if not _lib.on_gpu(device):
        return False
    try:
        _lib.load()
        return True
    except RuntimeError:
        return False


def quantizable(ggml_type: int, n_out: int, n_in: int, min_elements: int = 1 << 20) -> bool:
    """Kernel-capable; matrices smaller than `min_elements` stay bf16 (reference qlinear.py:46-52)."""
    name = GGML_TYPES[ggml_type][0]
    if name not in _QUANT:
        return False
    return n_in % FORMATS[name][0] == 0 and n_out > 0 and n_out * n_in >= min_elements


class QuantLinear:
    """y = x @ W^T (+ b) with W kept in its GGUF block format."""

    def __init__(self, raw: torch.Tensor, n_out: int, n_in: int, bias: Optional[torch.Tensor] = None,
                 type_name: str = ""):
        self.raw = raw
        self.n_out, self.n_in = n_out, n_in
        self.b = None if bias is None else bias.to(torch.bfloat16)
        self.type_name = type_name
        self.w = None   # duck typing with Linear (dtype queries)

    @property
    def dtype(self):
        return torch.bfloat16

    @property
    def mats(self):
        """The reference keeps tinygemm int4 tiles here (qlinear.py:200), which only its stacked-expert path
        reads (models/moe.py:56-80, torch._weight_int4pack_mm).  This QuantLinear keeps the GGUF bytes and has
        no int4 tiles: expert tensors load as PackedExperts instead (cudakern.IMMER_GEPACKT lists every
        format, so WeightLoader.experts takes that route), and asking for the tiles is an error."""
        raise RuntimeError("QuantLinear.mats: no int4 tile layout in this package (GGUF blocks are kept as they "
                           "are); expert tensors are PackedExperts here (cudakern.IMMER_GEPACKT)")

    def bf16_weight(self) -> torch.Tensor:
        """The matrix as (n_out, n_in) bf16 (reference qlinear.py:217-227), unpacked on the GPU."""
        return mmvq.entpacken(self.type_name, self.raw, self.n_out, self.n_in)

    def _mm(self, x2: torch.Tensor) -> torch.Tensor:
        return mmvq.mm(self.type_name, self.raw, x2, self.n_out, self.n_in)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, self.n_in)
        M = x2.shape[0]
        if M >= UNPACK_FROM:                     # long inputs: one unpack, one cuBLAS matmul (qlinear.py:232)
            y = x2.to(torch.bfloat16) @ self.bf16_weight().t()
        else:
            if x2.dtype != torch.float32:
                x2 = x2.to(torch.bfloat16)
            y = self._mm(x2).to(torch.bfloat16)
        if self.b is not None:
            y = y + self.b
        return y.reshape(*x.shape[:-1], self.n_out)


def build_quant_linear(raw: torch.Tensor, ggml_type: int, n_out: int, n_in: int,
                       bias: Optional[torch.Tensor] = None) -> QuantLinear:
    """raw: uint8 block bytes of an (n_out, n_in) GGUF matrix already on the CUDA device
    (reference qlinear.py:242-276)."""
    name, block_size, type_size = GGML_TYPES[ggml_type]
    if name not in _QUANT:
        raise GGUFError(f"{name} has no QuantLinear route in this path")
    if raw.numel() != n_out * n_in // block_size * type_size:
        raise GGUFError("byte count mismatch in build_quant_linear")
    if not _lib.on_gpu(raw):
        raise GGUFError("build_quant_linear: raw bytes must already be on the CUDA device")
    return QuantLinear(raw.reshape(-1).contiguous(), n_out, n_in, bias, name)
