"""Mixture-of-experts FFN on block-format experts, driven by router indices kept on the device.

    out[t] = sum_j w[t, j] * down_e(act(gate_e(x[t])) * up_e(x[t])),   e = idx[t, j]

Mirrors the reference's expert block for packed experts: routing as baukasten._auswahl
(ggufengine/models/baukasten.py:171-190, softmax gating, top-k, optional renormalisation) and the
graph-safe paths of moe.Experten.__call__ (ggufengine/models/moe.py:264-288: one token, and up to
GRAPH_ZEILEN tokens with every (token, slot) pair on its own).  Each token's input is quantised once
and read by all of its k slots (x_group = k); the down projection reads one activation row per slot.
Nothing reads the choice on the host, so a whole call can be captured in a CUDA graph.

With the default SiLU gate, experts resident on the device as contiguous tensors and gate and up in one
format, grouped_ffn (qmv_moe_ffn, up to MOE_MAX_PAIRS (token, slot) pairs and MOE_MAX_EXPERTS experts)
runs the FFN as one grouped launch sequence: quantise x; gate/up of every touched expert read once with
silu(g) * u quantised in its epilogue; down of every touched expert read once with the weighted sum
over slots in its epilogue.  MoeFFN uses it up to GROUPED_UP_TO pairs, where it is the faster of the two
(measured); above that, and otherwise, it runs expert matvecs per (token, slot) as above.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.nn.functional as F

from . import _lib
from .formats import TYPE_ID
from .layers import PackedExperts
from .mmvq import Eingang

GRAPH_ZEILEN = 16
MOE_MAX_PAIRS = 1024         # tokens x slots of one grouped call
MOE_MAX_EXPERTS = 1024       # experts of one grouped call
GROUPED_UP_TO = 16           # MoeFFN takes the grouped call up to this many pairs: measured at config 4 it
                             # beats the per-slot path at 8 pairs (batch 1) and loses from 32 (batch 4)


def grouped_ok(gate: PackedExperts, up: PackedExperts, down: PackedExperts, x: torch.Tensor, n_tok: int,
               k: int) -> bool:
    """True when grouped_ffn takes this call (SiLU gate assumed by the caller)."""
    return (1 <= n_tok and n_tok * k <= MOE_MAX_PAIRS and gate.n_exp <= MOE_MAX_EXPERTS and gate.name == up.name
            and all(ex.adressen is None and not ex.im_ram and _lib.on_gpu(ex.raw) for ex in (gate, up, down))
            and gate.raw.shape[1] == up.raw.shape[1] and x.device == down.raw.device and x.dim() == 2
            and x.stride(1) == 1 and gate.n_in % 32 == 0 and gate.n_out % 32 == 0)


def grouped_ffn(gate: PackedExperts, up: PackedExperts, down: PackedExperts, x: torch.Tensor, idx: torch.Tensor,
                w: torch.Tensor) -> torch.Tensor:
    """sum_j w[t, j] * down_e(silu(gate_e x_t) * up_e x_t) in three launches (qmv_moe_ffn).  x (L, dim)
    fp32 or bf16 with unit column stride (rows may be further apart), idx / w (L, k) -> (L, dim) float32.
    Raises where grouped_ok is false."""
    L, E = x.shape
    k = idx.shape[1]
    if not grouped_ok(gate, up, down, x, L, k):
        raise ValueError("grouped_ffn: shape, placement or expert count not supported")
    lib = _lib.load()
    ids = idx.reshape(-1).to(device=x.device, dtype=torch.int64).contiguous()
    wts = w.reshape(-1).to(device=x.device, dtype=torch.float32).contiguous()
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float().contiguous()
    n_ff = gate.n_out
    nbytes = lib.qmv_moe_workspace_bytes(L, k, E, n_ff)
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=x.device)
    off = (-ws.data_ptr()) % 256
    out = torch.empty(L, E, dtype=torch.float32, device=x.device)
    _lib.check(lib.qmv_moe_ffn(TYPE_ID[gate.name], _lib.ptr(gate.raw), _lib.ptr(up.raw), gate.raw.shape[1],
                               TYPE_ID[down.name], _lib.ptr(down.raw), down.raw.shape[1], gate.n_exp, _lib.ptr(ids),
                               _lib.ptr(wts), L, k, _lib.ptr(x), int(x.dtype == torch.float32), x.stride(0), E,
                               n_ff, ws.data_ptr() + off, _lib.ptr(out), _lib.stream_ptr(x.device)), "qmv_moe_ffn")
    return out


def route(logits: torch.Tensor, k: int, normalize: bool = True, weights_scale: float = 1.0):
    """Softmax router: (L, n_exp) logits -> (idx (L, k) int64, w (L, k) float32)."""
    p = torch.softmax(logits.float(), dim=-1)
    idx = p.topk(k, dim=-1)[1]
    w = p.gather(-1, idx)
    if normalize:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return idx, w * weights_scale


def _experts_mv(ex: PackedExperts, ids: torch.Tensor, e: Eingang, x_group: int) -> torch.Tensor:
    k = ids.numel()
    y = torch.empty(k, ex.n_out, dtype=torch.float32, device=ids.device)
    if ex.adressen is None:
        quelle, per = ex.raw, ex.raw.shape[1]
    else:
        quelle, per = ex.adressen, -1
    _lib.check(_lib.load().qmv_mv_experts(TYPE_ID[ex.name], _lib.ptr(quelle), per, ex.n_exp, _lib.ptr(ids), k,
                                          *e.zeiger(), x_group, _lib.ptr(y), ex.n_out, ex.n_in,
                                          _lib.stream_ptr(ids.device)), f"qmv_mv_experts {ex.name}")
    return y


class MoeFFN:
    """gate, up, down: PackedExperts of one layer.  act: elementwise activation (default SiLU)."""

    def __init__(self, gate: PackedExperts, up: PackedExperts, down: PackedExperts,
                 act: Optional[Callable[[torch.Tensor], torch.Tensor]] = None):
        if not (gate.n_exp == up.n_exp == down.n_exp):
            raise ValueError("expert counts differ between gate, up and down")
        if gate.n_out != up.n_out or down.n_in != gate.n_out or gate.n_in != down.n_out:
            raise ValueError("gate/up/down shapes do not chain")
        self.gate, self.up, self.down = gate, up, down
        self.act = act or F.silu
        self.n_exp = down.n_exp
        self.grouped = act is None or act is F.silu

    def _grouped_ok(self, x: torch.Tensor, L: int, k: int) -> bool:
        return self.grouped and L * k <= GROUPED_UP_TO and grouped_ok(self.gate, self.up, self.down, x, L, k)

    def grouped_call(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """The grouped launch sequence (grouped_ffn); raises where it does not apply."""
        if not self.grouped:
            raise ValueError("MoeFFN.grouped_call: the grouped kernels compute the SiLU gate only")
        return grouped_ffn(self.gate, self.up, self.down, x, idx, w)

    def __call__(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x (L, E) -> (L, E) float32; idx (L, k) expert ids, w (L, k) their weights."""
        L, E = x.shape
        k = idx.shape[1]
        if self._grouped_ok(x, L, k):
            return self.grouped_call(x, idx, w)
        ids = idx.reshape(-1).to(torch.int64).contiguous()
        ex = Eingang(x.float().contiguous())                        # L rows, one per token
        g = _experts_mv(self.gate, ids, ex, k)                      # (L*k, n_ff)
        u = _experts_mv(self.up, ids, ex, k)
        a = Eingang((self.act(g) * u).contiguous())                 # one row per (token, slot)
        y = _experts_mv(self.down, ids, a, 1)                       # (L*k, E)
        return (y.view(L, k, E) * w.float().unsqueeze(-1)).sum(1)
