"""Mixture-of-experts FFN on block-format experts, driven by router indices kept on the device.

    out[t] = sum_j w[t, j] * down_e(act(gate_e(x[t])) * up_e(x[t])),   e = idx[t, j]

Mirrors the reference's expert block for packed experts: routing as baukasten._auswahl
(ggufengine/models/baukasten.py:171-190, softmax gating, top-k, optional renormalisation) and the
graph-safe paths of moe.Experten.__call__ (ggufengine/models/moe.py:264-288: one token, and up to
GRAPH_ZEILEN tokens with every (token, slot) pair on its own).  Each token's input is quantised once
and read by all of its k slots (x_group = k); the down projection reads one activation row per slot.
Nothing reads the choice on the host, so a whole call can be captured in a CUDA graph.
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

    def __call__(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x (L, E) -> (L, E) float32; idx (L, k) expert ids, w (L, k) their weights."""
        L, E = x.shape
        k = idx.shape[1]
        ids = idx.reshape(-1).to(torch.int64).contiguous()
        ex = Eingang(x.float().contiguous())                        # L rows, one per token
        g = _experts_mv(self.gate, ids, ex, k)                      # (L*k, n_ff)
        u = _experts_mv(self.up, ids, ex, k)
        a = Eingang((self.act(g) * u).contiguous())                 # one row per (token, slot)
        y = _experts_mv(self.down, ids, a, 1)                       # (L*k, E)
        return (y.view(L, k, E) * w.float().unsqueeze(-1)).sum(1)
