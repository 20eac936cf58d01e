"""Drop-in for the reference's int8 matvec module (ggufengine/mmvq.py): the same names, argument
meaning and return shapes, computed by this package's sm_100a kernels through the C ABI.

* `Eingang` — the two-stage int8 activation input (mmvq.py:825-849), one quantisation per input,
  shared by every matrix that reads it.
* `mv` — y = W x for up to MMVQ_BIS tokens per call (mmvq.py:852-865), in launches of SPALTEN tokens,
  each weight byte read once per launch.
* `mm` — the reference's 17..112-token entry (mmvq.py:902-918); here the same int8 kernels in groups
  of SPALTEN tokens.
* `entpacken` — a block-format matrix unpacked to bf16 for long inputs (mmvq.py:931-940), every format.
* `norm_q8`, `akt_q8` — the fused one-token producers of an Eingang (mmvq.py:946-966): RMS norm with the
  residual add, and the gated activation, each one launch that also quantises its output.
* `mv_geteilt`, `mv_norm` (new) — up to four matrices on one single-token input in one launch;
  `mv_norm` forms norm_q8's RMS norm inside that launch (bit-identical to the two calls); with a
  `NextInput` the launch also forms the next matvec's input (quantised outputs, or SiLU·mul of two).
* `rope_kv`, `attention1`, `schritt_moeglich` — the attention steps of the reference's fused one-token
  layer (mmvq.py:969-1014) are not part of this package (the matvec path ends where attention begins).
  They are forwarded to an attention provider registered with `set_attention` (the reference's own
  module, for instance); without one `schritt_moeglich` is False and the reference's layer takes its
  general path, whose projections still run here through PackedLinear / mv.

Where the reference takes Q4_K and Q6_K only, these kernels take all twenty-six block formats of the path
(`FORMATE`: the classic, K-quant, IQ, MXFP4, ternary and 1-bit formats).  Everything runs on torch's current stream and is CUDA-graph
safe (no host reads, no synchronisation).  Non-CUDA tensors or unsupported formats raise; nothing
falls back to another implementation.
"""
from __future__ import annotations

import contextlib
import ctypes
import threading
from typing import Optional

import torch

from . import _lib
from .formats import FORMATS, TYPE_ID

FORMATE = dict(FORMATS)                 # name -> (values per block, bytes per block)
SPALTEN = 8                             # tokens per kernel launch (weights read once for all of them)
MMVQ_BIS = {f: 16 for f in FORMATE}     # up to this many tokens: mv (reference mmvq.py:32)
MMQ_BIS = {f: 112 for f in FORMATE}     # up to this many tokens: mm (reference mmvq.py:33)
SCHRITT_KERNE = ("quant_q8", "norm_q8", "akt_q8")   # fused one-token kernels of this package (mmvq.py:34)


def verfuegbar(device, fmt: str, n_in: int) -> bool:
    """Kernels for this format and row length on this device (reference mmvq.py:808-810)."""
    device = torch.device(device)
    if not _lib.on_gpu(device) or fmt not in FORMATE:
        return False
    return bool(_lib.load().qmv_supported(TYPE_ID[fmt], int(n_in)))


def _need_cuda(t: torch.Tensor, what: str) -> None:
    if not _lib.on_gpu(t):
        raise RuntimeError(f"{what}: tensor on {t.device}; the quantized matvec path runs on CUDA only")


class Eingang:
    """The int8 input of a vector — quantised once, read by every matrix that takes it
    (reference mmvq.py:825-849).  Without x only the buffers (a fused producer fills them)."""

    def __init__(self, x: Optional[torch.Tensor] = None, n: int = 0, device=None):
        if x is not None:
            _need_cuda(x, "Eingang")
            x = x.reshape(-1)
            if x.dtype != torch.float32:
                x = x.to(torch.bfloat16)
            x = x.contiguous()
            n, device = x.numel(), x.device
        if n % 32:
            raise ValueError(f"Eingang: {n} values is not a multiple of 32")
        self.n = n
        self.xq = torch.empty(n, dtype=torch.int8, device=device)
        self.xq2 = torch.empty(n, dtype=torch.int8, device=device)          # remainder, scale xd / 254
        self.xd = torch.empty(n // 32, dtype=torch.float32, device=device)
        self.xs = torch.empty(n // 32, dtype=torch.float32, device=device)
        if x is not None:
            _lib.check(_lib.load().qmv_quant_q8(_lib.ptr(x), int(x.dtype == torch.float32), *self.zeiger(), n,
                                                _lib.stream_ptr(x.device)), "qmv_quant_q8")

    def zeiger(self, ab: int = 0) -> list:
        """Pointers to xq, xq2, xd, xs from value `ab` on (the start of a row)."""
        if not ab:
            return [_lib.ptr(self.xq), _lib.ptr(self.xq2), _lib.ptr(self.xd), _lib.ptr(self.xs)]
        return [_lib.ptr(self.xq[ab:]), _lib.ptr(self.xq2[ab:]), _lib.ptr(self.xd[ab // 32:]),
                _lib.ptr(self.xs[ab // 32:])]


def _ist_eingang(x) -> bool:
    """An activation input: this module's Eingang or any object with its buffers (the reference's own
    Eingang, as its attention kernels return it, mmvq.py:987-1007)."""
    return isinstance(x, Eingang) or all(hasattr(x, a) for a in ("n", "xq", "xq2", "xd", "xs", "zeiger"))


def _check_raw(fmt: str, raw: torch.Tensor, n_out: int, n_in: int) -> None:
    _need_cuda(raw, f"mv {fmt}")
    if fmt not in FORMATE:
        raise RuntimeError(f"format {fmt} has no kernel in this path")
    bv, bb = FORMATE[fmt]
    if n_in % bv:
        raise RuntimeError(f"{fmt}: n_in {n_in} is not a multiple of {bv}")
    if raw.dtype != torch.uint8 or raw.numel() < n_out * (n_in // bv) * bb or not raw.is_contiguous():
        raise RuntimeError(f"{fmt}: raw must be contiguous uint8 with {n_out * (n_in // bv) * bb} bytes")


_PDL = [False]


def pdl(enabled: bool) -> bool:
    """Programmatic dependent launch for the single-token kernels and the activation producers (off by
    default; see include/nemicli_qmv.h, qmv_set_pdl): the next matvec streams its weights while the
    previous kernel finishes, a producer (quant_q8, norm_q8, akt_q8) launches while its input is still
    being written.  Only for weights that no kernel launched right before the matvec writes."""
    _PDL[0] = bool(enabled)
    return bool(_lib.load().qmv_set_pdl(int(bool(enabled))))


def _raw_x(x: torch.Tensor, n_in: int):
    """A one-token activation as the fused kernels take it (fp32 stays fp32, anything else bf16)."""
    x = x.reshape(-1)
    if x.numel() != n_in:
        return None
    if x.dtype != torch.float32:
        x = x.to(torch.bfloat16)
    return x.contiguous()


FUSED_MAX_IN = 8192     # without PDL: row length up to which quantising the input inside every CTA of
                        # the matvec beats a separate quantisation launch (measured: 4096 fused ahead
                        # by about 1 us, 14336 behind by 1.5-2.5 us).  With PDL the separate launch
                        # overlaps the previous kernel and is ahead at every length (2-2.5 us at 4096)


def _fused_ok(n_in: int) -> bool:
    return not _PDL[0] and n_in <= FUSED_MAX_IN


def _fused(fmt: str, mats, x: torch.Tensor, n_in: int, outs=None, force: bool = False):
    """One launch that quantises x itself; None where the staged kernel does not take the shape or
    the separate quantisation is faster (_fused_ok; unless force)."""
    if not (force or _fused_ok(n_in)):
        return None
    xr = _raw_x(x, n_in)
    if xr is None:
        return None
    _need_cuda(xr, f"mv {fmt}")
    dev = mats[0][0].device
    ys = outs or [torch.empty(n_out, dtype=torch.float32, device=dev) for _, n_out in mats]
    n = len(mats)
    w_arr = (ctypes.c_void_p * n)(*[raw.data_ptr() for raw, _ in mats])
    n_arr = (ctypes.c_int * n)(*[n_out for _, n_out in mats])
    y_arr = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
    st = _lib.load().qmv_mv_x(TYPE_ID[fmt], n, w_arr, n_arr, y_arr, n_in, _lib.ptr(xr),
                              int(xr.dtype == torch.float32), _lib.stream_ptr(dev))
    if st == 2:                       # row length the staged kernel does not take
        return None
    _lib.check(st, f"qmv_mv_x {fmt}")
    return ys


def mv(fmt: str, raw: torch.Tensor, x, n_out: int, n_in: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """raw: (n_out, n_in) in block format on the GPU; x: (M, n_in) or (n_in,) bf16/float32, or an
    Eingang with M rows -> (M, n_out) float32, or (n_out,) for a vector.  One token given as a tensor
    is quantised inside the matvec kernel (no separate Eingang) for rows up to FUSED_MAX_IN values when
    PDL is off.  out: a contiguous float32 tensor of M * n_out values to write into (this package's
    sharded layers gather from it in place)."""
    _check_raw(fmt, raw, n_out, n_in)
    ist_eingang = _ist_eingang(x)
    M = (x.n if ist_eingang else x.numel()) // n_in
    if out is not None and (out.dtype != torch.float32 or not out.is_contiguous() or out.numel() != M * n_out):
        raise RuntimeError(f"mv: out must be a contiguous float32 tensor of {M * n_out} values")
    if not ist_eingang and x.numel() == n_in:
        ys = _fused(fmt, [(raw, n_out)], x, n_in, None if out is None else [out.view(n_out)])
        if ys is not None:
            y = ys[0] if out is None else out
            return y.view(n_out) if x.dim() == 1 else y.view(1, n_out)
    e = x if ist_eingang else Eingang(x)
    if e.n % n_in:
        raise RuntimeError(f"mv: input of {e.n} values is not a whole number of rows of {n_in}")
    M = e.n // n_in
    y = torch.empty(M, n_out, dtype=torch.float32, device=raw.device) if out is None else out.view(M, n_out)
    _lib.check(_lib.load().qmv_mv(TYPE_ID[fmt], _lib.ptr(raw), n_out, n_in, *e.zeiger(), M, _lib.ptr(y),
                                  _lib.stream_ptr(raw.device)), f"qmv_mv {fmt}")
    vektor = M == 1 if ist_eingang else x.dim() == 1
    return y[0] if vektor else y


class NextInput:
    """The activation input of the next matvec, formed from a matvec's own outputs by the CTAs that
    write them (qmv_mv_multi_ep), so no producer launch follows the matvec: kind "quant" (one matrix's
    outputs quantised, as Eingang(y) would) or "silu_mul" (SiLU of one matrix's outputs times
    another's, as akt_q8(g, u, False) would; the fp32 product in `a`).  n: the values of the input.
    Holds the Eingang, `a` and one counter per 32 values (zero between calls).  Calls that share one
    object must not overlap on the GPU.  New entry point."""

    def __init__(self, n: int, kind: str, device):
        if kind not in ("quant", "silu_mul") or n % 32:
            raise ValueError(f"NextInput: kind quant or silu_mul and a multiple of 32 values (got {kind}, {n})")
        self.n, self.kind = n, kind
        self.eingang = Eingang(n=n, device=device)
        self.a = torch.empty(n, dtype=torch.float32, device=device) if kind == "silu_mul" else None
        self.counters = torch.zeros(n // 32, dtype=torch.int32, device=device)


def _produce(nxt: "NextInput", ys: list, src) -> None:
    """The producer launch that qmv_mv_multi_ep saves (the shapes it does not take)."""
    lib, e = _lib.load(), nxt.eingang
    y0 = ys[src[0]].reshape(-1)
    if nxt.kind == "quant":
        _lib.check(lib.qmv_quant_q8(_lib.ptr(y0), 1, *e.zeiger(), nxt.n, _lib.stream_ptr(y0.device)), "qmv_quant_q8")
    else:
        y1 = ys[src[1]].reshape(-1)
        _lib.check(lib.qmv_act_q8(_lib.ptr(y0), _lib.ptr(y1), 0, _lib.ptr(nxt.a), *e.zeiger(), nxt.n,
                                  _lib.stream_ptr(y0.device)), "qmv_act_q8")


def mv_geteilt(fmt: str, mats, x, n_in: int, next_input: Optional["NextInput"] = None, src=(0,)) -> list:
    """Several matrices that read the same input (q/k/v, gate/up) in one launch: mats = [(raw, n_out),
    ...] (at most 4); x one token ((n_in,) tensor or Eingang) -> [y (n_out,) float32, ...], or M tokens
    ((M, n_in) tensor or Eingang of M rows) -> [y (M, n_out), ...].  Each weight byte is read once per
    group of up to 8 tokens (Q4_K / Q8_0 several tokens: one tensor-core launch for all matrices); the
    input is quantised once.  next_input (one token): also form the next matvec's input from the
    outputs of matrices src (NextInput; in the same launch where the staged kernel takes it, else by
    the producer launch after it).  New entry point (the reference launches each matrix on its own)."""
    if not 1 <= len(mats) <= 4:
        raise RuntimeError("mv_geteilt: 1 to 4 matrices")
    for raw, n_out in mats:
        _check_raw(fmt, raw, n_out, n_in)
    if next_input is not None:
        need = 2 if next_input.kind == "silu_mul" else 1
        if len(src) != need or any(not 0 <= j < len(mats) or mats[j][1] != next_input.n for j in src):
            raise RuntimeError(f"mv_geteilt: next_input {next_input.kind} takes {need} matrices of {next_input.n} rows")
    if not _ist_eingang(x) and x.numel() == n_in and next_input is None:
        ys = _fused(fmt, mats, x, n_in)
        if ys is not None:
            return ys
    e = x if _ist_eingang(x) else Eingang(x)
    if e.n % n_in or e.n == 0:
        raise RuntimeError(f"mv_geteilt: rows of {n_in} values expected, got {e.n} values")
    M = e.n // n_in
    dev = mats[0][0].device
    ys = [torch.empty((n_out,) if M == 1 else (M, n_out), dtype=torch.float32, device=dev) for _, n_out in mats]
    n = len(mats)
    w_arr = (ctypes.c_void_p * n)(*[raw.data_ptr() for raw, _ in mats])
    n_arr = (ctypes.c_int * n)(*[n_out for _, n_out in mats])
    y_arr = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
    if next_input is not None:
        if M != 1:
            raise RuntimeError("mv_geteilt: next_input takes one token")
        nx = next_input
        st = _lib.load().qmv_mv_multi_ep(TYPE_ID[fmt], n, w_arr, n_arr, y_arr, n_in, *e.zeiger(),
                                         1 if nx.kind == "quant" else 2, src[0], src[-1], _lib.ptr(nx.counters),
                                         *nx.eingang.zeiger(), _lib.ptr(nx.a), _lib.stream_ptr(dev))
        if st != 2:
            _lib.check(st, f"qmv_mv_multi_ep {fmt}")
            return ys
    _lib.check(_lib.load().qmv_mv_multi_tok(TYPE_ID[fmt], n, w_arr, n_arr, y_arr, n_in, *e.zeiger(), M,
                                            _lib.stream_ptr(dev)), f"qmv_mv_multi_tok {fmt}")
    if next_input is not None:
        _produce(next_input, ys, src)
    return ys


def mv_norm(fmt: str, mats, h: torch.Tensor, w: torch.Tensor, eps: float, rest: Optional[torch.Tensor] = None,
            rs: float = 1.0, force: bool = False, next_input: Optional["NextInput"] = None, src=(0,)):
    """norm_q8(h, w, eps, rest, rs) followed by mv_geteilt on its input, in one launch: every CTA of the
    matvec forms the RMS norm (the norm kernel's sum order, so the quantised input and the outputs are
    bit-identical to the two calls).  mats = [(raw, n_out), ...] (1 to 4, one token) -> ([y (n_out,)
    float32, ...], new h) where new h = h + rs * rest (h itself without rest).  With PDL on (the two
    launches are faster then), for rows longer than FUSED_MAX_IN and for shapes the staged kernel does
    not take it is the two calls; force takes the one launch wherever the kernel takes the shape.
    next_input / src: as mv_geteilt (then always the two calls, the matvec forming the next input).
    New entry point (the reference's one-token step calls norm_q8 and then mv per matrix,
    models/baukasten.py:205-240)."""
    if not 1 <= len(mats) <= 4:
        raise RuntimeError("mv_norm: 1 to 4 matrices")
    hv, wv = _vektor(h, "mv_norm"), _vektor(w, "mv_norm")
    n_in = hv.numel()
    if rest is not None:
        rest = _vektor(rest, "mv_norm")
    if wv.numel() != n_in or (rest is not None and rest.numel() != n_in):
        raise RuntimeError(f"mv_norm: h, w and rest must have the same length ({n_in})")
    for raw, n_out in mats:
        _check_raw(fmt, raw, n_out, n_in)
    if next_input is None and (force or _fused_ok(n_in)):
        dev = mats[0][0].device
        ys = [torch.empty(n_out, dtype=torch.float32, device=dev) for _, n_out in mats]
        hn = None if rest is None else torch.empty(n_in, dtype=torch.float32, device=dev)
        n = len(mats)
        w_arr = (ctypes.c_void_p * n)(*[raw.data_ptr() for raw, _ in mats])
        n_arr = (ctypes.c_int * n)(*[n_out for _, n_out in mats])
        y_arr = (ctypes.c_void_p * n)(*[y.data_ptr() for y in ys])
        st = _lib.load().qmv_mv_norm(TYPE_ID[fmt], n, w_arr, n_arr, y_arr, n_in, _lib.ptr(hv), _lib.ptr(rest),
                                     ctypes.c_float(rs), _lib.ptr(hn), _lib.ptr(wv), ctypes.c_float(eps),
                                     _lib.stream_ptr(dev))
        if st != 2:
            _lib.check(st, f"qmv_mv_norm {fmt}")
            return ys, (h if hn is None else hn)
    _, e, h_new = norm_q8(h, w, eps, rest, rs)
    return mv_geteilt(fmt, mats, e, n_in, next_input, src), h_new


_TEILEN = threading.local()


@contextlib.contextmanager
def eingang_teilen():
    """Matrices with the same input (q/k/v, gate/up): inside this block an input tensor is quantised
    once (reference mmvq.py:871-879)."""
    alt = getattr(_TEILEN, "werte", None)
    _TEILEN.werte = {}
    try:
        yield
    finally:
        _TEILEN.werte = alt


def _eingang(x2: torch.Tensor) -> Eingang:
    geteilt = getattr(_TEILEN, "werte", None)
    schluessel = (x2.data_ptr(), tuple(x2.shape), x2.dtype)
    if geteilt is not None and schluessel in geteilt:
        return geteilt[schluessel][0]
    e = Eingang(x2)
    if geteilt is not None:
        geteilt[schluessel] = (e, x2)          # keep x2 alive while its address is a key
    return e


TC_FORMATE = ("Q4_K", "Q6_K")                # formats of the tensor-core tile path (the reference's MMQ)
TC_FROM = 48                                 # tokens from which the tile path beats the int8 kernels (measured),
TC_FROM_LARGE = 32                           # ... and for matrices of at least TC_LARGE weights
TC_LARGE = 32 * 2 ** 20


def tc_used(fmt: str, n_tok: int, n_out: int = 0, n_in: int = 0) -> bool:
    """Whether mm runs n_tok tokens of fmt (an n_out x n_in matrix) on the tensor-core tile path."""
    if fmt not in TC_FORMATE:
        return False
    return n_tok >= (TC_FROM_LARGE if n_out * n_in >= TC_LARGE else TC_FROM)


def mm(fmt: str, raw: torch.Tensor, x: torch.Tensor, n_out: int, n_in: int) -> torch.Tensor:
    """Several tokens: x (M, n_in) -> (M, n_out) float32 (reference mmvq.py:902-918).  Q4_K / Q6_K from
    TC_FROM tokens go to the tensor-core tile path with the reference MMQ's fp16 arithmetic (qmv_mm_tc);
    fewer tokens, the other formats and an Eingang input to the int8 kernels (faster there, and within
    the same tolerance of the exact product)."""
    _check_raw(fmt, raw, n_out, n_in)
    if not _ist_eingang(x) and tc_used(fmt, x.reshape(-1, n_in).shape[0], n_out, n_in):
        return mm_tc(fmt, raw, x, n_out, n_in)
    x2 = x.reshape(-1, n_in)
    e = _eingang(x2)
    M = x2.shape[0]
    y = torch.empty(M, n_out, dtype=torch.float32, device=raw.device)
    _lib.check(_lib.load().qmv_mv(TYPE_ID[fmt], _lib.ptr(raw), n_out, n_in, *e.zeiger(), M, _lib.ptr(y),
                                  _lib.stream_ptr(raw.device)), f"qmv_mv {fmt}")
    return y


def mm_tc(fmt: str, raw: torch.Tensor, x: torch.Tensor, n_out: int, n_in: int) -> torch.Tensor:
    """x (M, n_in) fp32 / bf16 -> (M, n_out) float32 on the tensor cores (Q4_K, Q6_K)."""
    _check_raw(fmt, raw, n_out, n_in)
    _need_cuda(x, "mm_tc input")
    if fmt not in TC_FORMATE:
        raise RuntimeError(f"mm_tc: {fmt} has no tensor-core tile path (Q4_K, Q6_K)")
    x2 = x.reshape(-1, n_in)
    if x2.dtype not in (torch.float32, torch.bfloat16):
        x2 = x2.float()
    x2 = x2.contiguous()
    M = x2.shape[0]
    lib = _lib.load()
    nbytes = lib.qmv_mm_tc_workspace_bytes(TYPE_ID[fmt], n_out, n_in, M)
    if nbytes <= 0:
        raise RuntimeError(f"mm_tc {fmt}: shape {n_out}x{n_in} not supported")
    ws = torch.empty(nbytes + 256, dtype=torch.uint8, device=raw.device)
    y = torch.empty(M, n_out, dtype=torch.float32, device=raw.device)
    _lib.check(lib.qmv_mm_tc(TYPE_ID[fmt], _lib.ptr(raw), n_out, n_in, _lib.ptr(x2), int(x2.dtype == torch.float32),
                             M, _lib.ptr(y), ws.data_ptr() + (-ws.data_ptr()) % 256, nbytes, _lib.stream_ptr(raw.device)),
               f"qmv_mm_tc {fmt}")
    return y


def block_sums(fmt: str, raw: torch.Tensor, e: Eingang, n_out: int, n_in: int):
    """Test hook: the int32 sums (code*xq, code*xq2) per row and unit of one token (include/nemicli_qmv.h)."""
    _check_raw(fmt, raw, n_out, n_in)
    unit = _lib.load().qmv_unit_values(TYPE_ID[fmt])        # the kernel's own unit: the buffers fit its writes
    s = torch.empty(n_out, n_in // unit, dtype=torch.int32, device=raw.device)
    s2 = torch.empty_like(s)
    _lib.check(_lib.load().qmv_block_sums(TYPE_ID[fmt], _lib.ptr(raw), n_out, n_in, _lib.ptr(e.xq), _lib.ptr(e.xq2),
                                          _lib.ptr(s), _lib.ptr(s2), _lib.stream_ptr(raw.device)),
               f"qmv_block_sums {fmt}")
    return s, s2


_OUT = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}


def entpacken(fmt: str, raw: torch.Tensor, n_out: int, n_in: int, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """raw: (n_out, n_in) in block format on the GPU -> (n_out, n_in) bf16 (reference mmvq.py:931-940), the
    reference's dequantised values rounded to nearest even (fp32 / fp16 with `dtype`)."""
    _check_raw(fmt, raw, n_out, n_in)
    if dtype not in _OUT:
        raise RuntimeError(f"entpacken: output dtype {dtype} (float32, bfloat16 or float16)")
    out = torch.empty(n_out, n_in, dtype=dtype, device=raw.device)
    _lib.check(_lib.load().qmv_unpack(TYPE_ID[fmt], _lib.ptr(raw), n_out * n_in, _lib.ptr(out), _OUT[dtype],
                                      _lib.stream_ptr(raw.device)), f"qmv_unpack {fmt}")
    return out


def _vektor(t: torch.Tensor, what: str) -> torch.Tensor:
    _need_cuda(t, what)
    if t.dtype != torch.float32 or not t.is_contiguous():
        raise RuntimeError(f"{what}: contiguous float32 vectors expected")
    return t.reshape(-1)


def norm_q8(h: torch.Tensor, w: torch.Tensor, eps: float, rest: Optional[torch.Tensor] = None, rs: float = 1.0):
    """RMS norm of one row; with `rest` first h = h + rs * rest.  -> (normalised float32, Eingang, new h)
    (reference mmvq.py:946-956).  One launch."""
    h_in = h
    h, w = _vektor(h, "norm_q8"), _vektor(w, "norm_q8")
    n = h.numel()
    e = Eingang(n=n, device=h.device)
    xn = torch.empty(n, dtype=torch.float32, device=h.device)
    hn = None
    if rest is not None:
        rest = _vektor(rest, "norm_q8")
        hn = torch.empty(n, dtype=torch.float32, device=h.device)
    _lib.check(_lib.load().qmv_norm_q8(_lib.ptr(h), _lib.ptr(rest), ctypes.c_float(rs), _lib.ptr(hn), _lib.ptr(w),
                                       ctypes.c_float(eps), _lib.ptr(xn), *e.zeiger(), n, _lib.stream_ptr(h.device)),
               "qmv_norm_q8")
    return xn, e, (h_in if hn is None else hn)


def akt_q8(g: torch.Tensor, u: Optional[torch.Tensor], gelu: bool):
    """act(g) * u (without u: act(g)), act = SiLU or GELU (tanh form) -> (float32, Eingang)
    (reference mmvq.py:959-966).  One launch."""
    g = _vektor(g, "akt_q8")
    n = g.numel()
    if u is not None:
        u = _vektor(u, "akt_q8")
    e = Eingang(n=n, device=g.device)
    a = torch.empty(n, dtype=torch.float32, device=g.device)
    _lib.check(_lib.load().qmv_act_q8(_lib.ptr(g), _lib.ptr(u), int(bool(gelu)), _lib.ptr(a), *e.zeiger(), n,
                                      _lib.stream_ptr(g.device)), "qmv_act_q8")
    return a, e


_ATTENTION = None


def set_attention(provider) -> None:
    """Registers the provider of the one-token attention steps (an object with rope_kv, attention1 and
    schritt_moeglich of the reference's signatures, e.g. the reference's own mmvq module); None removes it."""
    global _ATTENTION
    _ATTENTION = provider


def schritt_moeglich(device, H: int, Hkv: int, D: int) -> bool:
    """Can the reference's fused one-token layer step run (mmvq.py:1010-1014)?  Only with an attention
    provider that takes these head shapes; otherwise the layer takes its general path."""
    if _ATTENTION is None or not _lib.on_gpu(device):
        return False
    return bool(_ATTENTION.schritt_moeglich(device, H, Hkv, D))


def rope_kv(*args, **kwargs):
    """The provider's rope_kv (reference mmvq.py:969-984)."""
    if _ATTENTION is None:
        raise RuntimeError("rope_kv: no attention provider registered (mmvq.set_attention)")
    return _ATTENTION.rope_kv(*args, **kwargs)


def attention1(*args, **kwargs):
    """The provider's attention1 (reference mmvq.py:987-1007); its Eingang is read by mv directly."""
    if _ATTENTION is None:
        raise RuntimeError("attention1: no attention provider registered (mmvq.set_attention)")
    return _ATTENTION.attention1(*args, **kwargs)
