"""The reference's own callers on this package's mirrors (CPU, no GPU needed).

The reference's model code (ggufengine/models/common.py, moe.py, baukasten.py) is imported unchanged
from the reference tree with ggufengine.mmvq, ggufengine.cudakern and ggufengine.qlinear replaced by
this package's mirrors -- the swap INTEGRATION.md describes.  The CUDA library is replaced by a fake
that computes every entry point with the oracle on host memory (the tensors' data pointers are host
addresses here), and the mirrors' one device question (_lib.on_gpu) answers yes; the weight tensors
report is_cuda so that the reference's own dispatch takes its GPU branches.  What this checks: every
attribute and call the reference's callers make exists with the reference's meaning, the pointers the
mirrors pass are the right ones, and the results equal the oracle's.

Skipped where the reference tree is absent (it is only read here, never at run time).
"""
import ctypes
import os
import sys

import numpy as np
import pytest
import torch
import torch.nn.functional as F

REF = "/root/reference"
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "ggufengine")), reason="reference tree absent")

from nemicli_terminal_b200 import _lib, cudakern, layers, mmvq, qlinear, synth  # noqa: E402
from nemicli_terminal_b200.formats import FORMATS, TYPE_ID  # noqa: E402
from oracle import oracle as O  # noqa: E402


class Dev(torch.Tensor):
    """A host tensor that answers is_cuda: the reference's dispatch then takes its GPU branches."""

    @property
    def is_cuda(self):
        return True


def dev(t: torch.Tensor) -> torch.Tensor:
    return t.as_subclass(Dev)


def _addr(p):
    return p.value if isinstance(p, ctypes.c_void_p) else int(p or 0)


def _arr(p, dtype, n):
    a = _addr(p)
    if not a:
        return None
    return np.ctypeslib.as_array((ctypes.c_uint8 * (n * np.dtype(dtype).itemsize)).from_address(a)).view(dtype)


class FakeLib:
    """The C ABI computed by the oracle on host memory (include/nemicli_qmv.h meanings)."""

    def __init__(self):
        self.calls = []

    def _fmt(self, t):
        return {v: k for k, v in TYPE_ID.items()}[t]

    def qmv_supported(self, t, n_in):
        f = {v: k for k, v in TYPE_ID.items()}.get(t)
        return int(f is not None and n_in % FORMATS[f][0] == 0)

    def qmv_status_string(self, st):
        return b"fake status"

    def qmv_last_cuda_error(self):
        return 0

    def qmv_quant_q8(self, x, f32, xq, xq2, xd, xs, n, stream):
        self.calls.append("quant_q8")
        v = _arr(x, np.float32 if f32 else np.uint16, n).copy()
        q, q2, d, s = O.quant_q8(v)
        _arr(xq, np.int8, n)[:] = q
        _arr(xq2, np.int8, n)[:] = q2
        _arr(xd, np.float32, n // 32)[:] = d
        _arr(xs, np.float32, n // 32)[:] = s
        return 0

    def _eingang(self, xq, xq2, xd, xs, n):
        return (_arr(xq, np.int8, n).copy(), _arr(xq2, np.int8, n).copy(), _arr(xd, np.float32, n // 32).copy(),
                _arr(xs, np.float32, n // 32).copy())

    def qmv_mv(self, t, w, n_out, n_in, xq, xq2, xd, xs, n_tok, y, stream):
        self.calls.append(f"mv{n_tok}")
        fmt = self._fmt(t)
        raw = _arr(w, np.uint8, n_out * (n_in // FORMATS[fmt][0]) * FORMATS[fmt][1])
        ys = O.mv(fmt, raw, n_out, n_in, *self._eingang(xq, xq2, xd, xs, n_tok * n_in), n_tok=n_tok)
        _arr(y, np.float32, n_tok * n_out)[:] = ys.reshape(-1)
        return 0

    def qmv_mv_x(self, t, n_jobs, w, n_out, y, n_in, x, f32, stream):
        self.calls.append("mv_x")
        e = [np.zeros(n_in, np.int8), np.zeros(n_in, np.int8), np.zeros(n_in // 32, np.float32),
             np.zeros(n_in // 32, np.float32)]
        q = O.quant_q8(_arr(x, np.float32 if f32 else np.uint16, n_in).copy())
        fmt = self._fmt(t)
        rb = (n_in // FORMATS[fmt][0]) * FORMATS[fmt][1]
        for j in range(n_jobs):
            raw = _arr(w[j], np.uint8, n_out[j] * rb)
            _arr(y[j], np.float32, n_out[j])[:] = O.mv(fmt, raw, n_out[j], n_in, *q)[0]
        del e
        return 0

    def qmv_mv_experts(self, t, raw, per, n_exp, ids, k, xq, xq2, xd, xs, x_group, y, n_out, n_in, stream):
        self.calls.append("mv_experts")
        fmt = self._fmt(t)
        rb = (n_in // FORMATS[fmt][0]) * FORMATS[fmt][1]
        idv = _arr(ids, np.int64, k).copy()
        rows = (k + x_group - 1) // x_group if x_group > 1 else k
        e = self._eingang(xq, xq2, xd, xs, rows * n_in)
        out = _arr(y, np.float32, k * n_out)
        for j in range(k):
            r = j // x_group
            base = _addr(raw) + int(idv[j]) * per if per >= 0 else int(_arr(raw, np.int64, n_exp)[idv[j]])
            wj = _arr(ctypes.c_void_p(base), np.uint8, n_out * rb)
            ej = [e[0][r * n_in:(r + 1) * n_in], e[1][r * n_in:(r + 1) * n_in], e[2][r * n_in // 32:(r + 1) * n_in // 32],
                  e[3][r * n_in // 32:(r + 1) * n_in // 32]]
            out[j * n_out:(j + 1) * n_out] = O.mv(fmt, wj, n_out, n_in, *ej)[0]
        return 0

    def qmv_unpack(self, t, w, n, out, dt, stream):
        self.calls.append("unpack")
        fmt = self._fmt(t)
        raw = _arr(w, np.uint8, n // FORMATS[fmt][0] * FORMATS[fmt][1])
        v = torch.from_numpy(O.dequant(fmt, raw.copy(), n))
        tgt = {0: torch.float32, 1: torch.bfloat16, 2: torch.float16}[dt]
        bits = v.to(tgt).view(torch.int32 if dt == 0 else torch.int16).numpy()
        _arr(out, bits.dtype, n)[:] = bits
        return 0

    def qmv_norm_q8(self, h, r, rs, hout, w, eps, xn, xq, xq2, xd, xs, n, stream):
        self.calls.append("norm_q8")
        v = _arr(h, np.float32, n).copy()
        if _addr(r):
            v = (v + np.float32(rs.value) * _arr(r, np.float32, n)).astype(np.float32)
            _arr(hout, np.float32, n)[:] = v
        inv = np.float32(1.0 / np.sqrt(np.mean(v.astype(np.float64) ** 2) + eps.value))
        x = (v * inv * _arr(w, np.float32, n)).astype(np.float32)
        _arr(xn, np.float32, n)[:] = x
        q = O.quant_q8(x)
        for p, a in zip((xq, xq2, xd, xs), q):
            _arr(p, a.dtype, a.size)[:] = a
        return 0

    def qmv_act_q8(self, g, u, gelu, a, xq, xq2, xd, xs, n, stream):
        self.calls.append("act_q8")
        gv = torch.from_numpy(_arr(g, np.float32, n).copy())
        v = F.gelu(gv, approximate="tanh") if gelu else F.silu(gv)
        if _addr(u):
            v = v * torch.from_numpy(_arr(u, np.float32, n).copy())
        v = v.numpy().astype(np.float32)
        _arr(a, np.float32, n)[:] = v
        q = O.quant_q8(v)
        for p, arr in zip((xq, xq2, xd, xs), q):
            _arr(p, arr.dtype, arr.size)[:] = arr
        return 0


@pytest.fixture
def ref(monkeypatch):
    """The reference's model modules, imported with this package's mirrors in place of its kernel modules."""
    fake = FakeLib()
    monkeypatch.setattr(_lib, "load", lambda: fake)
    monkeypatch.setattr(_lib, "on_gpu", lambda x: True)
    monkeypatch.setattr(_lib, "stream_ptr", lambda device=None: ctypes.c_void_p(0))
    saved = {k: v for k, v in sys.modules.items() if k == "ggufengine" or k.startswith("ggufengine.")}
    for k in saved:
        del sys.modules[k]
    monkeypatch.syspath_prepend(REF)
    sys.modules["ggufengine.mmvq"] = mmvq
    sys.modules["ggufengine.cudakern"] = cudakern
    sys.modules["ggufengine.qlinear"] = qlinear
    import ggufengine.models.baukasten as baukasten
    import ggufengine.models.common as common
    import ggufengine.models.moe as moe
    yield {"common": common, "moe": moe, "baukasten": baukasten, "fake": fake}
    for k in [k for k in sys.modules if k == "ggufengine" or k.startswith("ggufengine.")]:
        del sys.modules[k]
    sys.modules.update(saved)


def _lin(common, fmt, n_out, n_in, seed, cls=None):
    raw = dev(synth.blocks(fmt, n_out, n_in, seed=seed))
    return (cls or common.PackedLinear)(raw, TYPE_ID[fmt], n_out, n_in, None, torch.float32), raw


def _oracle_a(fmt, raw, n_out, n_in, x):
    return O.mv_exact(fmt, np.asarray(raw.as_subclass(torch.Tensor)), n_out, n_in, x.numpy().reshape(-1, n_in))


@pytest.mark.parametrize("mirror", [False, True])
def test_baukasten_one_token_path(ref, mirror):
    """_schritt's matvec calls: norm_q8 -> _int8_weg / _mal(q) -> akt_q8 -> _mal(down)."""
    common, bk = ref["common"], ref["baukasten"]
    cls = layers.PackedLinear if mirror else None
    if mirror:                                     # this package's PackedLinear in the reference's module
        bk.PackedLinear = layers.PackedLinear
    q, qraw = _lin(common, "Q4_K", 96, 512, 1, cls)
    down, draw = _lin(common, "Q6_K", 512, 256, 2, cls)
    assert bk._int8_weg(q) and bk._int8_weg(down)     # reads lin.mmvq, lin.band, lin.im_ram
    assert q.band is None and q.nr == -1 and q.mm_bis == cudakern.MM_ZEILEN and not q.im_ram
    h = torch.randn(512)
    w = torch.rand(512) + 0.5
    xn, e, h2 = mmvq.norm_q8(h, w, 1e-5)
    assert h2 is h and e.n == 512
    yq = bk._mal(q, e, xn)
    assert yq.shape == (96,)
    assert O.max_rel(yq.numpy(), _oracle_a("Q4_K", qraw, 96, 512, xn)) < 1e-3
    g = torch.randn(256)
    u = torch.randn(256)
    a, ea = mmvq.akt_q8(g, u, False)
    assert torch.allclose(a, F.silu(g) * u, rtol=1e-6, atol=1e-7)
    yd = bk._mal(down, ea, a)
    assert O.max_rel(yd.numpy(), _oracle_a("Q6_K", draw, 512, 256, a)) < 1e-3
    assert {"norm_q8", "act_q8", "mv1"} <= set(ref["fake"].calls)
    bk.PackedLinear = common.PackedLinear


@pytest.mark.parametrize("mirror", [False, True])
@pytest.mark.parametrize("M", [1, 4, 20, 200])
def test_packed_linear_rechnen(ref, mirror, M):
    """PackedLinear._rechnen for one token, a few, MMQ_BIS range and the unpack + matmul range."""
    common = ref["common"]
    lin, raw = _lin(common, "IQ2_XXS", 64, 256, 3, layers.PackedLinear if mirror else None)
    x = torch.randn(M, 256)
    y = lin(x)
    assert y.shape == (M, 64)
    ya = _oracle_a("IQ2_XXS", raw, 64, 256, x)
    tol = 2e-2 if M > 112 else 1e-3                # long inputs: bf16 unpacked weights and inputs, as the reference
    assert O.max_rel(y.numpy(), ya) < tol
    want = "unpack" if M > 112 else ("mv_x" if M == 1 else "mv")
    assert any(c.startswith(want) for c in ref["fake"].calls)


def _experts(common, fmt, n_exp, n_out, n_in, seed, cls):
    raw = dev(synth.blocks(fmt, n_exp * n_out, n_in, seed=seed))
    return cls(raw, TYPE_ID[fmt], n_exp, n_out, n_in, torch.float32)


@pytest.mark.parametrize("mirror", [False, True])
@pytest.mark.parametrize("L", [1, 4, 20])
def test_moe_experten(ref, mirror, L):
    """moe._teil picks _GepacktTeil for packed experts; Experten.__call__ for one token (graph-safe ids),
    a few tokens (per-pair path) and longer inputs (sorted groups through PackedExperts.weights)."""
    common, moe = ref["common"], ref["moe"]
    cls = layers.PackedExperts if mirror else common.PackedExperts
    if mirror:
        moe.PackedExperts = layers.PackedExperts
    n_exp, E, n_ff, k = 8, 256, 64, 2
    gate = _experts(common, "Q4_K", n_exp, n_ff, E, 10, cls)
    up = _experts(common, "Q4_K", n_exp, n_ff, E, 11, cls)
    down = _experts(common, "Q4_0", n_exp, E, n_ff, 12, cls)
    teile = [moe._teil(t) for t in (gate, up, down)]
    assert all(isinstance(t, moe._GepacktTeil) for t in teile)
    ex = moe.Experten.__new__(moe.Experten)
    ex.akt, ex.glu, ex.gate_up = F.silu, None, None
    ex.gate, ex.up, ex.down = teile
    ex.n_exp, ex.bias, ex.lager = n_exp, {}, None
    ex.graphfaehig = all(t.graphfaehig for t in teile)
    x = torch.randn(L, E)
    if L == 4:                                     # the graph-capture branch: every (token, slot) pair on its own
        moe.mehrere_aufnahme = lambda: True
        x = dev(x)
    idx = torch.stack([torch.randperm(n_exp)[:k] for _ in range(L)])
    w = torch.rand(L, k)
    out = ex(x, idx, w)
    assert out.shape == (L, E)
    # dense fp64 reference with the dequantised experts and the unquantised activations
    ref_out = torch.zeros(L, E, dtype=torch.float64)
    deq = lambda t, e, n_out, n_in: torch.from_numpy(O.dequant(t.name, np.asarray(t.raw[e].as_subclass(torch.Tensor)),  # noqa: E731
                                                               n_out * n_in)).view(n_out, n_in).double()
    for t_ in range(L):
        for j in range(k):
            e = int(idx[t_, j])
            a = F.silu(deq(gate, e, n_ff, E) @ x[t_].double()) * (deq(up, e, n_ff, E) @ x[t_].double())
            ref_out[t_] += float(w[t_, j]) * (deq(down, e, E, n_ff) @ a)
    assert O.max_rel(out.as_subclass(torch.Tensor).double().numpy(), ref_out.numpy()) < 1e-3
    moe.mehrere_aufnahme = common.mehrere_aufnahme
    if mirror:
        moe.PackedExperts = common.PackedExperts
        assert (L == 20) == ("unpack" in ref["fake"].calls)      # only the sorted path unpacks


def test_loader_routes_experts_to_packed(ref):
    """WeightLoader's expert route: packed_type() reads cudakern.IMMER_GEPACKT, which lists every format
    here, so expert tensors of any format stay PackedExperts (never the int4 QuantLinear stack)."""
    common = ref["common"]
    for fmt in FORMATS:
        assert common.packed_type(TYPE_ID[fmt])
    ql = qlinear.build_quant_linear(dev(synth.blocks("Q8_0", 32, 256, seed=1)), TYPE_ID["Q8_0"], 32, 256)
    with pytest.raises(RuntimeError, match="int4"):
        ql.mats
    w = ql.bf16_weight()
    assert w.dtype == torch.bfloat16 and w.shape == (32, 256)
    assert cudakern._nvrtc_pfad() is not None               # schichten.int8_weg_da: the int8 path exists
