"""Decode chain: a decode step's dependent matvec stages in one persistent launch (qmv_chain).

The reference's fused one-token layer step (ggufengine/models/baukasten.py:217-240) runs, per layer,
norm_q8 -> mv(q), mv(k), mv(v) -> rope/attention -> mv(o) -> norm_q8 -> mv(gate), mv(up) -> akt_q8 ->
mv(down): about a dozen launches, each paying launch and pipeline-fill latency.  Here the matvec stages
of many layers run in one cooperative kernel: each stage's input is produced inside the kernel (RMS norm
with the residual add, SiLU gate, or a plain vector), CTAs meet at a grid barrier only where a stage reads
earlier outputs, and the weight stream never stops at those barriers.  Attention sits outside this path;
a caller that has it splits the chain around it.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List, Optional, Sequence

import torch

from . import _lib
from .formats import TYPE_ID

RAW, RMSNORM, SILU_MUL = 0, 1, 2
MAX_STAGES = 128


class _Stage(ctypes.Structure):
    """Mirror of qmv_stage (include/nemicli_qmv.h)."""
    _fields_ = [
        ("ggml_type", ctypes.c_int),
        ("n_jobs", ctypes.c_int),
        ("w", ctypes.c_void_p * 4),
        ("n_out", ctypes.c_int * 4),
        ("y", ctypes.c_void_p * 4),
        ("n_in", ctypes.c_int),
        ("input", ctypes.c_int),
        ("a", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("norm_w", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("h_out", ctypes.c_void_p),
        ("wait", ctypes.c_int),
    ]


@dataclass
class Stage:
    """Matrices [(raw, n_out), ...] of one format and row length that read the input built from a/b."""
    fmt: str
    mats: Sequence[tuple]
    n_in: int
    input: int = RAW
    a: Optional[torch.Tensor] = None
    b: Optional[torch.Tensor] = None
    norm_w: Optional[torch.Tensor] = None
    eps: float = 1e-5
    h_out: Optional[torch.Tensor] = None
    wait: bool = True
    ys: List[torch.Tensor] = field(default_factory=list)


def _p(t) -> Optional[int]:
    return None if t is None else t.data_ptr()


class Chain:
    """A fixed list of stages with their output buffers; `run()` enqueues the whole chain (graph safe)."""

    def __init__(self, stages: Sequence[Stage], device=None):
        if not 1 <= len(stages) <= MAX_STAGES:
            raise RuntimeError(f"chain: 1..{MAX_STAGES} stages")
        dev = torch.device(device) if device is not None else stages[0].mats[0][0].device
        if dev.type != "cuda":
            raise RuntimeError("chain: CUDA only (no CPU fallback)")
        self.stages = list(stages)
        self.arr = (_Stage * len(stages))()
        for s, st in zip(self.arr, self.stages):
            if not 1 <= len(st.mats) <= 4:
                raise RuntimeError("chain: 1..4 matrices per stage")
            for t in (st.a, st.b, st.norm_w):
                if t is not None and (t.dtype != torch.float32 or not t.is_contiguous() or t.numel() != st.n_in):
                    raise RuntimeError(f"chain: stage inputs must be contiguous fp32 vectors of {st.n_in}")
            if not st.ys:
                st.ys = [torch.empty(n_out, dtype=torch.float32, device=dev) for _, n_out in st.mats]
            s.ggml_type = TYPE_ID[st.fmt]
            s.n_jobs = len(st.mats)
            for j, (raw, n_out) in enumerate(st.mats):
                s.w[j] = raw.data_ptr()
                s.n_out[j] = n_out
                s.y[j] = st.ys[j].data_ptr()
            s.n_in = st.n_in
            s.input = st.input
            s.a, s.b, s.norm_w, s.h_out = _p(st.a), _p(st.b), _p(st.norm_w), _p(st.h_out)
            s.eps = st.eps
            s.wait = int(st.wait)
        self.workspace = torch.zeros(_lib.load().qmv_chain_workspace_bytes(), dtype=torch.uint8, device=dev)
        self.device = dev

    def run(self) -> None:
        _lib.check(_lib.load().qmv_chain(self.arr, len(self.stages), _lib.ptr(self.workspace),
                                         _lib.stream_ptr(self.device)), "qmv_chain")


def layer_stages(q, k, v, o, gate, up, down, h_in: torch.Tensor, resid_in: Optional[torch.Tensor],
                 attn_norm: torch.Tensor, ffn_norm: torch.Tensor, eps: float = 1e-5, first: bool = False):
    """The four matvec stages of a Llama-style layer around a residual stream.

    q..down: (fmt, raw, n_out, n_in).  h_in (+ resid_in when given) is the residual stream entering the
    layer.  The attention output that o_proj reads is stood in for by q_proj's output (attention is
    outside this path).  Returns (stages, h_mid, y_down): h_mid = h + resid after the attention block's
    residual add is written by the FFN stage; the next layer takes (h_mid, y_down)."""
    dev = h_in.device
    n = h_in.numel()
    h_attn = torch.empty(n, dtype=torch.float32, device=dev) if resid_in is not None else None
    s1 = Stage(q[0], [(q[1], q[2]), (k[1], k[2]), (v[1], v[2])], q[3], RMSNORM, a=h_in, b=resid_in,
               norm_w=attn_norm, eps=eps, h_out=h_attn, wait=not first)
    s1.ys = [torch.empty(m[2], dtype=torch.float32, device=dev) for m in (q, k, v)]
    s2 = Stage(o[0], [(o[1], o[2])], o[3], RAW, a=s1.ys[0], wait=True)
    s2.ys = [torch.empty(o[2], dtype=torch.float32, device=dev)]
    h_base = h_attn if h_attn is not None else h_in
    h_mid = torch.empty(n, dtype=torch.float32, device=dev)
    s3 = Stage(gate[0], [(gate[1], gate[2]), (up[1], up[2])], gate[3], RMSNORM, a=h_base, b=s2.ys[0],
               norm_w=ffn_norm, eps=eps, h_out=h_mid, wait=True)
    s3.ys = [torch.empty(m[2], dtype=torch.float32, device=dev) for m in (gate, up)]
    s4 = Stage(down[0], [(down[1], down[2])], down[3], SILU_MUL, a=s3.ys[0], b=s3.ys[1], wait=True)
    s4.ys = [torch.empty(down[2], dtype=torch.float32, device=dev)]
    return [s1, s2, s3, s4], h_mid, s4.ys[0]
