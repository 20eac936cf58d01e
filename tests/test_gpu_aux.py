"""The kernels around the matvecs on the GPU: unpacking (qmv_unpack: mmvq.entpacken, PackedExperts.weights,
QuantLinear.bf16_weight, PackedLinear's long-input path) and the fused one-token producers (qmv_norm_q8,
qmv_act_q8: mmvq.norm_q8, mmvq.akt_q8), and the norm fused into the matvec (qmv_mv_norm: mmvq.mv_norm,
bit-identical to norm_q8 followed by the matvecs).

Unpacking is bit-exact: its fp32 values against the reference's own dequantised golden vectors
(tests/golden, every format and every codebook entry), bf16 / fp16 against torch's round-to-nearest-even
of those.  The producers against torch fp32 (1e-6), and their activation input bit-exact against the
oracle's quantisation of the kernel's own normalised / activated output."""
import ctypes
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from nemicli_terminal_b200 import _lib, layers, mmvq, qlinear, synth
from nemicli_terminal_b200.formats import FORMATS, TYPE_ID
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "dequant_golden.npz"))
KEYS = sorted({k.split("__")[0] for k in GOLDEN.files})
NAME = {v: k for k, v in O.TYPES.items()}


@pytest.mark.parametrize("key", KEYS)
def test_unpack_bit_exact_with_reference_golden(cuda, key):
    t, rows, cols = (int(v) for v in GOLDEN[key + "__shape"])
    fmt = NAME[t]
    raw = torch.from_numpy(GOLDEN[key + "__raw"].copy()).to(cuda)
    deq = torch.from_numpy(GOLDEN[key + "__deq"].copy()).view(rows, cols)
    y32 = mmvq.entpacken(fmt, raw, rows, cols, torch.float32).cpu()
    assert torch.equal(y32.view(torch.int32), deq.view(torch.int32)), fmt
    for dt in (torch.bfloat16, torch.float16):
        y = mmvq.entpacken(fmt, raw, rows, cols, dt).cpu()
        assert torch.equal(y.view(torch.int16), deq.to(dt).view(torch.int16)), (fmt, dt)


@pytest.mark.parametrize("fmt", sorted(FORMATS))
def test_unpack_large_matches_oracle(cuda, fmt):
    n_out, n_in = 1024, 4096
    raw = synth.blocks(fmt, n_out, n_in, seed=5)
    ref = torch.from_numpy(O.dequant(fmt, raw.numpy(), n_out * n_in)).view(n_out, n_in)
    y = mmvq.entpacken(fmt, raw.to(cuda), n_out, n_in).cpu()
    assert torch.equal(y.view(torch.int16), ref.to(torch.bfloat16).view(torch.int16))


def test_unpack_refusals(cuda):
    from nemicli_terminal_b200 import _lib
    L = _lib.load()
    raw = synth.blocks("Q4_K", 4, 256, seed=1).to(cuda)
    out = torch.empty(4, 256, device=cuda)
    assert L.qmv_unpack(99, _lib.ptr(raw), 1024, _lib.ptr(out), 0, None) == 1          # unknown format
    assert L.qmv_unpack(TYPE_ID["Q4_K"], _lib.ptr(raw), 1000, _lib.ptr(out), 0, None) == 2   # not whole blocks
    assert L.qmv_unpack(TYPE_ID["Q4_K"], _lib.ptr(raw), 1024, _lib.ptr(out), 7, None) == 2   # no such dtype
    assert L.qmv_unpack(TYPE_ID["Q4_K"], _lib.ptr(raw), 1024, _lib.ptr(out[0, 1:]), 0, None) == 3  # misaligned


def test_packed_experts_weights_and_items(cuda):
    n_exp, n_out, n_in = 6, 64, 512
    raw = synth.blocks("IQ2_XXS", n_exp * n_out, n_in, seed=7)
    ex = layers.PackedExperts(raw.to(cuda), TYPE_ID["IQ2_XXS"], n_exp, n_out, n_in, torch.bfloat16)
    ids = torch.tensor([4, 1, 4], device=cuda)
    w = ex.weights(ids)
    assert w.shape == (3, n_out, n_in) and w.dtype == torch.bfloat16
    for j, e in enumerate((4, 1, 4)):
        ref = torch.from_numpy(O.dequant("IQ2_XXS", raw.view(n_exp, -1)[e].numpy(), n_out * n_in)).view(n_out, n_in)
        assert torch.equal(w[j].cpu().view(torch.int16), ref.to(torch.bfloat16).view(torch.int16))
    x = synth.activations(3, n_in, seed=1, device=cuda).to(torch.bfloat16)
    y = ex[1](x)
    assert torch.allclose(y.float(), (x @ w[1].t()).float())
    with pytest.raises(IndexError):
        ex[n_exp]


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K", "IQ3_S"])
def test_packed_linear_long_inputs_unpack(cuda, fmt):
    """M > MMQ_BIS: the unpack + cuBLAS route of PackedLinear._rechnen (reference common.py:414-428)."""
    n_out, n_in, M = 512, 1024, 200
    raw = synth.blocks(fmt, n_out, n_in, seed=9)
    pl = layers.PackedLinear(raw.to(cuda), TYPE_ID[fmt], n_out, n_in, None, torch.bfloat16)
    x = synth.activations(M, n_in, seed=2, device=cuda)
    y = pl(x).float().cpu()
    w = torch.from_numpy(O.dequant(fmt, raw.numpy(), n_out * n_in)).view(n_out, n_in).to(torch.bfloat16)
    ref = (x.cpu().to(torch.bfloat16).double() @ w.double().t())
    assert O.max_rel(y.numpy(), ref.numpy()) < 1e-2           # bf16 output, as the reference


def test_quant_linear_bf16_weight(cuda):
    raw = synth.blocks("Q8_0", 256, 512, seed=4)
    ql = qlinear.build_quant_linear(raw.to(cuda), TYPE_ID["Q8_0"], 256, 512)
    w = ql.bf16_weight().cpu()
    ref = torch.from_numpy(O.dequant("Q8_0", raw.numpy(), 256 * 512)).view(256, 512).to(torch.bfloat16)
    assert torch.equal(w.view(torch.int16), ref.view(torch.int16))
    x = synth.activations(300, 512, seed=3, device=cuda)       # M >= UNPACK_FROM: unpack + cuBLAS
    y = ql(x).float().cpu()
    assert O.max_rel(y.numpy(), (x.cpu().to(torch.bfloat16).double() @ ref.double().t()).numpy()) < 1e-2


def _eingang_matches_oracle(e, v):
    q, q2, d, s = O.quant_q8(v.cpu().numpy())
    assert np.array_equal(e.xq.cpu().numpy(), q) and np.array_equal(e.xq2.cpu().numpy(), q2)
    assert np.array_equal(e.xd.cpu().numpy(), d) and np.array_equal(e.xs.cpu().numpy(), s)


@pytest.mark.parametrize("n", [512, 4096, 14336])
@pytest.mark.parametrize("rest", [False, True])
def test_norm_q8(cuda, n, rest):
    h = synth.activations(1, n, seed=n, device=cuda)[0]
    w = torch.rand(n, device=cuda) + 0.5
    r = synth.activations(1, n, seed=n + 1, device=cuda)[0] if rest else None
    xn, e, h2 = mmvq.norm_q8(h, w, 1e-5, rest=r, rs=0.5 if rest else 1.0)
    v = h + 0.5 * r if rest else h
    if rest:
        assert torch.equal(h2, v)
    else:
        assert h2 is h
    ref = v * torch.rsqrt(v.pow(2).mean() + 1e-5) * w
    assert float((xn - ref).abs().max() / ref.abs().max()) < 1e-6
    _eingang_matches_oracle(e, xn)
    y = mmvq.mv("Q4_K", synth.blocks("Q4_K", 64, n, seed=3, device=cuda), e, 64, n)
    assert y.shape == (64,)


@pytest.mark.parametrize("gelu", [False, True])
@pytest.mark.parametrize("with_u", [False, True])
def test_akt_q8(cuda, gelu, with_u):
    n = 14336
    g = synth.activations(1, n, seed=1, device=cuda)[0] * 3
    u = synth.activations(1, n, seed=2, device=cuda)[0] if with_u else None
    a, e = mmvq.akt_q8(g, u, gelu)
    ref = F.gelu(g, approximate="tanh") if gelu else F.silu(g)
    if with_u:
        ref = ref * u
    assert float((a - ref).abs().max() / ref.abs().max()) < 1e-6
    _eingang_matches_oracle(e, a)


@pytest.mark.parametrize("fmt,n,force", [("Q4_K", 4096, False), ("Q8_0", 4096, False), ("IQ2_XXS", 2048, False),
                                         ("Q6_K", 14336, True), ("Q6_K", 14336, False), ("Q4_0", 14336 + 256, True),
                                         ("Q4_K", 4096, True)])
@pytest.mark.parametrize("rest", [False, True])
@pytest.mark.parametrize("pdl", [False, True])
def test_mv_norm_equals_two_calls(cuda, fmt, n, force, rest, pdl):
    """mv_norm (the RMS norm formed by every CTA of the matvec) gives the quantised input of norm_q8 and
    so the same outputs, bit for bit, with one and several matrices, with and without the residual add
    (scaled); the new h equals norm_q8's.  Without force and with PDL on, or past FUSED_MAX_IN, it is
    the two calls (launched with PDL when it is on)."""
    old = mmvq.pdl(pdl)
    try:
        h = synth.activations(1, n, seed=n, device=cuda)[0]
        w = torch.rand(n, device=cuda) + 0.5
        r = synth.activations(1, n, seed=n + 1, device=cuda)[0] if rest else None
        rs = 0.75 if rest else 1.0
        mats = [(synth.blocks(fmt, n_out, n, seed=5 + n_out, device=cuda), n_out) for n_out in (512, 128, 256)]
        ys, h_new = mmvq.mv_norm(fmt, mats, h, w, 1e-5, rest=r, rs=rs, force=force)
        _, e, h_ref = mmvq.norm_q8(h, w, 1e-5, rest=r, rs=rs)
        ref = mmvq.mv_geteilt(fmt, mats, e, n)
        assert all(torch.equal(a, b) for a, b in zip(ys, ref))
        assert torch.equal(h_new, h_ref) if rest else h_new is h
        y1, _ = mmvq.mv_norm(fmt, mats[:1], h, w, 1e-5, rest=r, rs=rs, force=force)
        assert torch.equal(y1[0], ref[0])
    finally:
        mmvq.pdl(old)


def test_mv_norm_refusals(cuda):
    lib = _lib.load()
    h = torch.zeros(4096, device=cuda)
    w = torch.ones(4096, device=cuda)
    raw = synth.blocks("Q4_K", 64, 4096, seed=1, device=cuda)
    y = torch.empty(64, device=cuda)
    wa = (ctypes.c_void_p * 1)(raw.data_ptr())
    na = (ctypes.c_int * 1)(64)
    ya = (ctypes.c_void_p * 1)(y.data_ptr())

    def st(*a):
        return lib.qmv_mv_norm(TYPE_ID["Q4_K"], *a)
    one, eps = ctypes.c_float(1.0), ctypes.c_float(1e-5)
    assert st(1, wa, na, ya, 4096, _lib.ptr(h), None, one, None, None, eps, None) == 6          # no norm weights
    assert st(1, wa, na, ya, 4096, _lib.ptr(h), _lib.ptr(h), one, None, _lib.ptr(w), eps, None) == 6   # r, no h_out
    assert st(5, wa, na, ya, 4096, _lib.ptr(h), None, one, None, _lib.ptr(w), eps, None) == 4    # > 4 matrices
    assert st(1, wa, na, ya, 4000, _lib.ptr(h), None, one, None, _lib.ptr(w), eps, None) == 2    # row length


def _eingang_equal(a, b):
    return all(torch.equal(getattr(a, f), getattr(b, f)) for f in ("xq", "xq2", "xd", "xs"))


@pytest.mark.parametrize("fmt,n_in,rows,kind", [
    ("Q4_K", 4096, (4096, 1024, 1024), "quant"),       # q/k/v: o's input from q
    ("Q4_K", 4096, (14336, 14336), "silu_mul"),         # gate/up: down's input
    ("Q8_0", 4096, (512, 256), "quant"),
    ("Q6_K", 14336, (2048, 2048), "silu_mul"),
    ("Q4_K", 1024, (512, 512), "silu_mul"),             # narrow teams: the producer launch instead
])
@pytest.mark.parametrize("pdl", [False, True])
def test_next_input_equals_producers(cuda, fmt, n_in, rows, kind, pdl):
    """mv_geteilt with a NextInput: the outputs are those of the plain call, and the next input formed
    by the CTAs that finish each 32-row group equals, bit for bit, Eingang(y) ("quant") or akt_q8(g, u)
    ("silu_mul"), on two calls in a row with different inputs (the group counters reset themselves)."""
    old = mmvq.pdl(pdl)
    try:
        mats = [(synth.blocks(fmt, n, n_in, seed=31 + j, device=cuda), n) for j, n in enumerate(rows)]
        src = (0,) if kind == "quant" else (0, 1)
        nxt = mmvq.NextInput(rows[0], kind, cuda)
        for call in range(2):
            e = mmvq.Eingang(synth.activations(1, n_in, seed=40 + call, device=cuda)[0].contiguous())
            ys = mmvq.mv_geteilt(fmt, mats, e, n_in, next_input=nxt, src=src)
            ref = mmvq.mv_geteilt(fmt, mats, e, n_in)
            assert all(torch.equal(a, b) for a, b in zip(ys, ref))
            if kind == "quant":
                assert _eingang_equal(nxt.eingang, mmvq.Eingang(ys[0]))
            else:
                a, e2 = mmvq.akt_q8(ys[0], ys[1], False)
                assert torch.equal(nxt.a, a) and _eingang_equal(nxt.eingang, e2)
            assert int(nxt.counters.abs().sum()) == 0
    finally:
        mmvq.pdl(old)


def test_next_input_refusals(cuda):
    e = mmvq.Eingang(synth.activations(1, 4096, seed=1, device=cuda)[0].contiguous())
    mats = [(synth.blocks("Q4_K", 512, 4096, seed=2, device=cuda), 512)]
    with pytest.raises(RuntimeError):                                     # silu_mul needs two matrices
        mmvq.mv_geteilt("Q4_K", mats, e, 4096, next_input=mmvq.NextInput(512, "silu_mul", cuda), src=(0,))
    with pytest.raises(RuntimeError):                                     # rows differ from the input's size
        mmvq.mv_geteilt("Q4_K", mats, e, 4096, next_input=mmvq.NextInput(1024, "quant", cuda), src=(0,))
    with pytest.raises(ValueError):
        mmvq.NextInput(100, "quant", cuda)
