"""The linear-op boundary of the reference's model code (ggufengine/models/common.py): PackedLinear
(:364-431) and PackedExperts (:434-492), the objects its loader creates for weights that stay in
GGUF block format.  Same constructor arguments and call signatures; the computation is this
package's int8 kernels for every token count (the reference switches between its int8 kernels,
MMQ, float kernels and unpack + cuBLAS).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import cudakern, mmvq
from .formats import GGML_TYPES


class PackedLinear:
    """y = x @ W^T (+ b), W (n_out, n_in) kept in a block format."""

    def __init__(self, raw: torch.Tensor, ggml_type: int, n_out: int, n_in: int,
                 bias: Optional[torch.Tensor], dtype: torch.dtype):
        self.raw = raw.view(1, -1)
        self.ggml_type = ggml_type
        self.n_out, self.n_in = n_out, n_in
        self.b = None if bias is None else bias.to(dtype)
        self.dtype = dtype
        self.w = None                            # duck typing with Linear
        self.name = GGML_TYPES[ggml_type][0]
        _, bs, ts = GGML_TYPES[ggml_type]
        self.zeilen_bytes = n_in // bs * ts
        self.mmvq = raw.is_cuda and mmvq.verfuegbar(raw.device, self.name, n_in)
        self.kernel = self.mmvq
        if not self.mmvq:
            raise RuntimeError(f"PackedLinear: no kernel for {self.name} (n_in {n_in}) on {raw.device}")

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, self.n_in)
        M = x2.shape[0]
        if M <= mmvq.MMVQ_BIS[self.name]:
            y = mmvq.mv(self.name, self.raw, x2, self.n_out, self.n_in)
        else:
            y = mmvq.mm(self.name, self.raw, x2, self.n_out, self.n_in)
        y = y.to(self.dtype)
        if self.b is not None:
            y = y + self.b
        return y.reshape(*x.shape[:-1], self.n_out)


class PackedExperts:
    """Expert tensor (n_expert, out, in) kept in its GGUF block format; the chosen experts are
    multiplied directly on the block data, ids staying on the device."""

    def __init__(self, raw: torch.Tensor, ggml_type: int, n_exp: int, n_out: int, n_in: int,
                 dtype: torch.dtype, geraet: Optional[torch.device] = None):
        self.raw = raw.view(n_exp, -1)
        self.geraet = torch.device(geraet) if geraet is not None else raw.device
        self.ggml_type = ggml_type
        self.n_exp, self.n_out, self.n_in = n_exp, n_out, n_in
        self.dtype = dtype
        self.name = GGML_TYPES[ggml_type][0]
        self.kernel = raw.is_cuda and cudakern.verfuegbar(self.geraet, self.name, n_in)
        if not self.kernel:
            raise RuntimeError(f"PackedExperts: no kernel for {self.name} (n_in {n_in}) on {self.geraet}")
        self.im_ram = False
        self.adressen: Optional[torch.Tensor] = None   # optional address table (one int64 per expert)

    def __len__(self) -> int:
        return self.n_exp

    def matvec(self, ids: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """The experts `ids` (k,) applied to one shared input x (n_in,) -> (k, n_out) float32."""
        return cudakern.mv(self.name, self.raw, ids, x.reshape(-1), self.n_out, self.n_in, self.adressen)

    def matvec_je(self, ids: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
        """Expert ids[j] applied to its own input a[j]: (k, n_in) -> (k, n_out) float32."""
        return cudakern.mv(self.name, self.raw, ids, a.reshape(ids.numel(), -1), self.n_out, self.n_in,
                           self.adressen)
