"""Grouped expert matvec, the linear-op boundary objects and the MoE FFN on the GPU.

Mirrors the reference's kernel tests (tests/test_gguf_iq.py:207-256 there): ids [4, 0, 2] with a
shared and a per-expert input, an odd row count, CUDA-graph replay with changed ids; plus an
address table, refused ids, PackedLinear / QuantLinear / PackedExperts and the MoE FFN."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from nemicli_terminal_b200 import _lib, cudakern, layers, moe, qlinear, synth
from nemicli_terminal_b200.formats import FORMATS, TYPE_ID, row_bytes
from oracle import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu


def _experts(fmt, n_exp, n_out, n_in, seed):
    raw = synth.blocks(fmt, n_exp * n_out, n_in, seed=seed)
    return raw.view(n_exp, -1)


def _ref(fmt, raw_e, n_out, n_in, x):
    """oracle B per expert: raw_e (n_out*row bytes,), x (n_in,) fp32/bf16 -> (n_out,) fp64."""
    y, _ = H.oracle_b(fmt, raw_e.reshape(-1), x.reshape(1, -1), n_out, n_in)
    return y[0]


@pytest.mark.parametrize("fmt", H.FMTS)
def test_expert_gather(cuda, fmt):
    n_in = 768 if FORMATS[fmt][0] > 32 else 96
    raw = _experts(fmt, 5, 12, n_in, seed=4)               # 12 rows: the last row group is half full
    ids = torch.tensor([4, 0, 2])
    x = synth.activations(1, n_in, seed=5)[0].to(torch.bfloat16)
    y = cudakern.mv(fmt, raw.to(cuda), ids.to(cuda), x.to(cuda), 12, n_in).cpu().numpy()
    for j, e in enumerate(ids.tolist()):
        assert O.max_rel(y[j], _ref(fmt, raw[e], 12, n_in, x)) < 1e-5
    a = synth.activations(3, n_in, seed=6).to(torch.bfloat16)     # each expert its own input
    y = cudakern.mv(fmt, raw.to(cuda), ids.to(cuda), a.to(cuda), 12, n_in).cpu().numpy()
    for j, e in enumerate(ids.tolist()):
        assert O.max_rel(y[j], _ref(fmt, raw[e], 12, n_in, a[j])) < 1e-5


def test_address_table(cuda):
    fmt, n_in = "Q4_K", 512
    raw = _experts(fmt, 4, 16, n_in, seed=8).to(cuda)
    spare = [r.clone() for r in raw]                       # experts somewhere else in memory
    table = torch.tensor([s.data_ptr() for s in spare], dtype=torch.int64, device=cuda)
    ids = torch.tensor([3, 1], device=cuda)
    x = synth.activations(1, n_in, seed=9, device=cuda)[0]
    y_tab = cudakern.mv(fmt, raw, ids, x, 16, n_in, adressen=table)
    y_raw = cudakern.mv(fmt, raw, ids, x, 16, n_in)
    assert torch.equal(y_tab, y_raw)


def test_refused_ids_give_zeros_and_flag(cuda):
    fmt, n_in = "Q4_K", 256
    raw = _experts(fmt, 3, 8, n_in, seed=1).to(cuda)
    _lib.device_status(clear=True)
    ids = torch.tensor([0, 7, -3, 2], device=cuda)
    x = synth.activations(1, n_in, seed=2, device=cuda)[0]
    y = cudakern.mv(fmt, raw, ids, x, 8, n_in)
    assert _lib.device_status(clear=True) & 1
    assert (y[1] == 0).all() and (y[2] == 0).all()
    ok = cudakern.mv(fmt, raw, torch.tensor([0, 2], device=cuda), x, 8, n_in)
    assert torch.equal(y[0], ok[0]) and torch.equal(y[3], ok[1])
    assert _lib.device_status(clear=True) == 0


@pytest.mark.parametrize("n_in", [256, 4096])
def test_padding_slots_give_zeros_without_flag(cuda, n_in):
    """Expert id -1 marks an unused slot of a padded exchange buffer: zero rows, no error bit
    (256: fallback kernel, 4096: staged kernel)."""
    fmt = "Q4_K"
    raw = _experts(fmt, 3, 64, n_in, seed=3).to(cuda)
    _lib.device_status(clear=True)
    x = synth.activations(1, n_in, seed=4, device=cuda)[0]
    y = cudakern.mv(fmt, raw, torch.tensor([1, -1, -1, 2], device=cuda), x, 64, n_in)
    assert _lib.device_status(clear=True) == 0
    assert (y[1] == 0).all() and (y[2] == 0).all()
    ok = cudakern.mv(fmt, raw, torch.tensor([1, 2], device=cuda), x, 64, n_in)
    assert torch.equal(y[0], ok[0]) and torch.equal(y[3], ok[1])


def test_cuda_graph_replay_with_new_ids(cuda):
    fmt, n_in = "IQ2_XXS", 512
    raw = _experts(fmt, 3, 8, n_in, seed=6).to(cuda)
    ids = torch.tensor([2, 1], device=cuda)
    x = synth.activations(1, n_in, seed=7, device=cuda)[0].to(torch.bfloat16)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        cudakern.mv(fmt, raw, ids, x, 8, n_in)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = cudakern.mv(fmt, raw, ids, x, 8, n_in)
    ids.copy_(torch.tensor([0, 2]))                        # new choice, same graph
    g.replay()
    torch.cuda.synchronize()
    want = cudakern.mv(fmt, raw, torch.tensor([0, 2], device=cuda), x, 8, n_in)
    assert torch.equal(y, want)


@pytest.mark.parametrize("fmt", H.FMTS)
def test_packed_linear_routes(cuda, fmt):
    n_out, n_in = 96, 512 if FORMATS[fmt][0] > 32 else 160
    raw, _ = H.case(fmt, n_out, n_in, seed=12)
    pl = layers.PackedLinear(raw.to(cuda), TYPE_ID[fmt], n_out, n_in, None, torch.bfloat16)
    for M in (1, 9, 20, 40):
        x = synth.activations(M, n_in, seed=M).to(torch.bfloat16)
        y = pl(x.to(cuda)).float().cpu().numpy()
        ya = H.oracle_a(fmt, raw, x, n_out, n_in)
        assert y.shape == (M, n_out)
        assert O.max_rel(y, ya) < 1e-2            # bf16 output rounding (the reference casts too)


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0"])
def test_quant_linear(cuda, fmt):
    n_out, n_in = 512, 1024
    raw, _ = H.case(fmt, n_out, n_in, seed=13)
    bias = torch.randn(n_out)
    ql = qlinear.build_quant_linear(raw.to(cuda), TYPE_ID[fmt], n_out, n_in, bias.to(cuda))
    assert ql.dtype == torch.bfloat16
    x = synth.activations(5, n_in, seed=1).to(torch.bfloat16)
    y = ql(x.to(cuda)).float().cpu().numpy()
    ya = H.oracle_a(fmt, raw, x, n_out, n_in) + bias.numpy()
    assert O.max_rel(y, ya) < 1e-2


@pytest.mark.parametrize("L", [1, 4, 16])
def test_moe_ffn(cuda, L):
    n_exp, k, E, n_ff = 16, 4, 512, 256
    mk = lambda n_out, n_in, seed: layers.PackedExperts(              # noqa: E731
        _experts("Q4_K", n_exp, n_out, n_in, seed).to(cuda), TYPE_ID["Q4_K"], n_exp, n_out, n_in, torch.bfloat16)
    gate, up, down = mk(n_ff, E, 1), mk(n_ff, E, 2), mk(E, n_ff, 3)
    ffn = moe.MoeFFN(gate, up, down)
    x = synth.activations(L, E, seed=L, device=cuda)
    idx, w = moe.route(synth.router_logits(L, n_exp, seed=L, device=cuda), k)
    out = ffn(x, idx, w)
    # reference: dense fp64 per (token, slot) with the dequantised experts
    Wg = [torch.from_numpy(O.dequant("Q4_K", gate.raw[e].cpu().numpy(), n_ff * E)).view(n_ff, E).double() for e in range(n_exp)]
    Wu = [torch.from_numpy(O.dequant("Q4_K", up.raw[e].cpu().numpy(), n_ff * E)).view(n_ff, E).double() for e in range(n_exp)]
    Wd = [torch.from_numpy(O.dequant("Q4_K", down.raw[e].cpu().numpy(), n_ff * E)).view(E, n_ff).double() for e in range(n_exp)]
    xc, ic, wc = x.cpu().double(), idx.cpu(), w.cpu().double()
    ref = torch.zeros(L, E, dtype=torch.float64)
    for t in range(L):
        for j in range(k):
            e = int(ic[t, j])
            a = F.silu(Wg[e] @ xc[t]) * (Wu[e] @ xc[t])
            ref[t] += wc[t, j] * (Wd[e] @ a)
    assert O.max_rel(out.cpu().numpy(), ref.numpy()) < 1e-3
    assert torch.equal(out, ffn(x, idx, w))                # run to run (the reference's test_moe.py:80)


@pytest.mark.parametrize("fmt", H.FMTS)
def test_shared_input_launch(cuda, fmt):
    """mv_geteilt: q/k/v-like matrices sharing one input, one launch == separate launches (bit for bit)."""
    from nemicli_terminal_b200 import mmvq
    n_in = 4096
    shapes = [512, 128, 128] if fmt != "Q8_0" else [256, 64]
    raws = [synth.blocks(fmt, n, n_in, seed=i).to(cuda) for i, n in enumerate(shapes)]
    x = synth.activations(1, n_in, seed=3, device=cuda)[0]
    e = mmvq.Eingang(x)
    ys = mmvq.mv_geteilt(fmt, list(zip(raws, shapes)), e, n_in)
    for raw, n, y in zip(raws, shapes, ys):
        assert torch.equal(y, mmvq.mv(fmt, raw, e, n, n_in))
