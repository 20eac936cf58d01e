"""Drop-in for the reference's per-format block kernels (ggufengine/cudakern.py) for the seven block
formats of this path: the expert gather `mv` driven by device-side ids (cudakern.py:756-774) and the
few-row `mm` (cudakern.py:777-790).

The reference computes these in fp32 from a bf16 copy of x; here x is quantised once into the
two-stage int8 input and the kernels take integer dot products (see mmvq.Eingang).  fp32 inputs are
quantised from fp32, anything else from bf16 (as the reference converts, cudakern.py:765).
Everything is CUDA-graph safe: ids stay on the device and are never read on the host.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from .formats import FORMATS, TYPE_ID
from .mmvq import Eingang

FORMATE = dict(FORMATS)
# Formats that always stay in block format (cudakern.py:52-54).  The reference lists those without an int4
# QuantLinear route; here no format is repacked, so every format of this path is listed, and the reference's
# loader keeps expert tensors of any of them as PackedExperts (models/common.py:280-282, 220-224).
IMMER_GEPACKT = frozenset(FORMATE)
MM_ZEILEN = 16                                    # rows of one `mm` call (cudakern.py:31)


_cu = None


def _treiber():
    """The CUDA driver library (reference cudakern.py:586-596; hostmem.py maps pinned memory through it)."""
    global _cu
    if _cu is None:
        import ctypes
        cu = ctypes.CDLL("libcuda.so.1")
        cu.cuLaunchKernel.argtypes = [ctypes.c_void_p] + [ctypes.c_uint] * 6 + [
            ctypes.c_uint, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        _cu = cu
    return _cu


def _nvrtc_pfad():
    """Where the kernels come from (reference cudakern.py:580-583 returns the NVRTC library, whose presence
    tells schichten.int8_weg_da that the int8 path exists): here the prebuilt kernel library, or None."""
    try:
        _lib.load()
    except RuntimeError:
        return None
    return _lib.lib_path()


def verfuegbar(device, fmt: str, n_in: int) -> bool:
    """Kernel for this format and row length on this device (cudakern.py:733-739)."""
    device = torch.device(device)
    if not _lib.on_gpu(device) or fmt not in FORMATE:
        return False
    return bool(_lib.load().qmv_supported(TYPE_ID[fmt], int(n_in)))


def mm_bis(device) -> int:
    """Most input rows of one `mm` call on this device (cudakern.py:742-745)."""
    return MM_ZEILEN if _lib.on_gpu(device) else 1


def _eingang(x: torch.Tensor) -> Eingang:
    return Eingang(x if x.dtype == torch.float32 else x.to(torch.bfloat16))


def mv(fmt: str, raw: torch.Tensor, ids: torch.Tensor, x: torch.Tensor, n_out: int, n_in: int,
       adressen: Optional[torch.Tensor] = None) -> torch.Tensor:
    """raw (n_exp, bytes per expert) on the GPU; ids (k,) expert ids on the GPU.  x (n_in,) is shared by
    all chosen experts, x (k, n_in) is each expert's own input.  adressen (n_exp,) int64 on the GPU:
    where each expert's bytes lie (then raw is not read).  -> (k, n_out) float32."""
    if fmt not in FORMATE:
        raise RuntimeError(f"format {fmt} has no kernel in this path")
    if not _lib.on_gpu(x):
        raise RuntimeError("cudakern.mv: x must be on the GPU (no CPU fallback)")
    geraet = x.device
    ids = ids.to(geraet, torch.int64).contiguous()
    k = ids.numel()
    je = x.dim() == 2
    if je and x.shape[0] != k:
        raise RuntimeError(f"cudakern.mv: {x.shape[0]} inputs for {k} experts")
    e = _eingang(x.reshape(-1))
    y = torch.empty(k, n_out, dtype=torch.float32, device=geraet)
    if adressen is None:
        raw2 = raw.reshape(raw.shape[0], -1) if raw.dim() > 1 else raw.view(1, -1)
        if not _lib.on_gpu(raw2):
            raise RuntimeError("cudakern.mv: expert bytes must be device-addressable (GPU memory)")
        quelle, per, n_exp = raw2, raw2.shape[1], raw2.shape[0]
    else:
        quelle, per, n_exp = adressen.to(geraet, torch.int64).contiguous(), -1, adressen.numel()
    _lib.check(_lib.load().qmv_mv_experts(TYPE_ID[fmt], _lib.ptr(quelle), per, n_exp, _lib.ptr(ids), k,
                                          *e.zeiger(), 1 if je else k, _lib.ptr(y), n_out, n_in,
                                          _lib.stream_ptr(geraet)), f"qmv_mv_experts {fmt}")
    return y


def mm(fmt: str, raw: torch.Tensor, x: torch.Tensor, n_out: int, n_in: int) -> torch.Tensor:
    """raw: one matrix (n_out rows) in block format on the GPU, x (M, n_in) with 2 <= M <= mm_bis
    -> (M, n_out) float32; every weight is read once for all rows (cudakern.py:777-790)."""
    M = x.shape[0]
    if not 2 <= M <= mm_bis(x.device):
        raise ValueError(f"mm: {M} rows (2..{mm_bis(x.device)})")
    if fmt not in FORMATE:
        raise RuntimeError(f"format {fmt} has no kernel in this path")
    if not (_lib.on_gpu(raw) and _lib.on_gpu(x)):
        raise RuntimeError("cudakern.mm: tensors must be on the GPU (no CPU fallback)")
    e = _eingang(x.reshape(-1))
    y = torch.empty(M, n_out, dtype=torch.float32, device=x.device)
    _lib.check(_lib.load().qmv_mv(TYPE_ID[fmt], _lib.ptr(raw), n_out, n_in, *e.zeiger(), M, _lib.ptr(y),
                                  _lib.stream_ptr(x.device)), f"qmv_mv {fmt}")
    return y
