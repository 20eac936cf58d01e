"""The linear-op boundary of the reference's model code (ggufengine/models/common.py): PackedLinear
(:364-431) and PackedExperts (:434-492), the objects its loader creates for weights that stay in
GGUF block format.  Same constructor arguments, attributes and call signatures, so the reference's
callers (baukasten._mal / _int8_weg, WeightLoader.linear, moe._GepacktTeil, Fliessband) use them
unchanged; the computation is this package's kernels: the int8 matvec for up to MMQ_BIS tokens, and
for longer inputs the matrix unpacked on the GPU (qmv_unpack) and multiplied by cuBLAS, as the
reference does.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib, cudakern, mmvq
from .formats import GGML_TYPES


class PackedLinear:
    """y = x @ W^T (+ b), W (n_out, n_in) kept in a block format."""

    KERNEL_BIS = cudakern.MM_ZEILEN
    ZEILEN_JE_STUECK = 32 * 1024 * 1024          # values unpacked at once (reference common.py:369)

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
        self.kernel = _lib.on_gpu(raw) and cudakern.verfuegbar(raw.device, self.name, n_in)
        self.mmvq = _lib.on_gpu(raw) and mmvq.verfuegbar(raw.device, self.name, n_in)
        if not self.mmvq:
            raise RuntimeError(f"PackedLinear: no kernel for {self.name} (n_in {n_in}) on {raw.device}")
        self.mm_bis = min(self.KERNEL_BIS, cudakern.mm_bis(raw.device)) if self.kernel else 1
        # pinned host memory mapped for the GPU (the reference's hostmem.abgebildet): set by a loader that
        # places the bytes there; the int8 kernels then stay off this matrix, as in the reference
        self.im_ram = False
        self.band = None                         # a Fliessband: whole copies a few matrices ahead
        self.nr = -1
        self._nullen: dict = {}

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if self.band is None:
            return self._rechnen(x, self.raw)
        roh = self.band.holen(self.nr).view(1, -1)
        try:
            return self._rechnen(x, roh)
        finally:
            self.band.fertig(self.nr)

    def _rechnen(self, x: torch.Tensor, raw: torch.Tensor) -> torch.Tensor:
        """The reference's dispatch (common.py:400-431): up to MMVQ_BIS / MMQ_BIS tokens the int8 kernels,
        longer inputs row chunks unpacked to the compute dtype and multiplied by cuBLAS."""
        x2 = x.reshape(-1, self.n_in)
        M = x2.shape[0]
        im_ram = self.im_ram and raw is self.raw
        if _lib.on_gpu(raw) and M <= mmvq.MMVQ_BIS[self.name] and not im_ram:
            y = mmvq.mv(self.name, raw, x2, self.n_out, self.n_in).to(self.dtype)
        elif _lib.on_gpu(raw) and M <= mmvq.MMQ_BIS[self.name] and not im_ram:
            y = mmvq.mm(self.name, raw, x2, self.n_out, self.n_in).to(self.dtype)
        else:
            xd = x2.to(self.dtype)
            y = torch.empty(M, self.n_out, dtype=self.dtype, device=x2.device)
            stueck = max(1, self.ZEILEN_JE_STUECK // self.n_in)
            for r0 in range(0, self.n_out, stueck):
                r1 = min(r0 + stueck, self.n_out)
                roh = raw[0, r0 * self.zeilen_bytes:r1 * self.zeilen_bytes]
                if im_ram:                       # one copy over PCIe; unpacking reads the bytes several times
                    roh = roh.to(x2.device)
                w = mmvq.entpacken(self.name, roh, r1 - r0, self.n_in).to(self.dtype)
                y[:, r0:r1] = xd @ w.t()
                del w
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
        lesbar = _lib.on_gpu(raw) or (_lib.on_gpu(self.geraet) and raw.is_pinned())
        self.kernel = lesbar and cudakern.verfuegbar(self.geraet, self.name, n_in)
        if not self.kernel:
            raise RuntimeError(f"PackedExperts: no kernel for {self.name} (n_in {n_in}) on {self.geraet}")
        self.im_ram = not _lib.on_gpu(raw) and _lib.on_gpu(self.geraet) and raw.is_pinned()
        self.adressen: Optional[torch.Tensor] = None   # optional address table (one int64 per expert)

    def __len__(self) -> int:
        return self.n_exp

    def weights(self, ids: torch.Tensor) -> torch.Tensor:
        """(k,) expert ids (any device) -> (k, n_out, n_in) in the compute dtype (reference common.py:456-460):
        the chosen experts' bytes gathered on the GPU and unpacked there (qmv_unpack)."""
        part = self.raw.index_select(0, ids.to(self.raw.device)).to(self.geraet, non_blocking=True)
        k = part.shape[0]
        w = mmvq.entpacken(self.name, part.reshape(-1), k * self.n_out, self.n_in,
                           self.dtype if self.dtype in (torch.float32, torch.float16) else torch.bfloat16)
        return w.to(self.dtype).view(k, self.n_out, self.n_in)

    def matvec(self, ids: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        """The experts `ids` (k,) applied to one shared input x (n_in,) -> (k, n_out) float32."""
        return cudakern.mv(self.name, self.raw, ids, x.reshape(-1), self.n_out, self.n_in, self.adressen)

    def matvec_je(self, ids: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
        """Expert ids[j] applied to its own input a[j]: (k, n_in) -> (k, n_out) float32."""
        return cudakern.mv(self.name, self.raw, ids, a.reshape(ids.numel(), -1), self.n_out, self.n_in,
                           self.adressen)

    def __getitem__(self, e: int) -> "_PackedExpert":
        if not 0 <= e < self.n_exp:
            raise IndexError(e)
        return _PackedExpert(self, e)


class _PackedExpert:
    """One expert of a PackedExperts tensor as a linear layer (reference common.py:483-492)."""

    def __init__(self, owner: PackedExperts, e: int):
        self.owner, self.e = owner, e
        self.n_out, self.n_in = owner.n_out, owner.n_in

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        w = self.owner.weights(torch.tensor([self.e], device=self.owner.geraet))[0]
        return x.to(w.dtype) @ w.t()
