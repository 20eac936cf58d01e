"""The grouped MoE FFN (qmv_moe_ffn: quantise, gate/up with the SiLU product, down with the weighted
slot sum) on the GPU.

Checked against the per-(token, slot) expert path (qmv_mv_experts, pinned to the oracle in
test_gpu_experts.py) in every format, against a dense fp64 restatement of the reference's
Experten.__call__ (ggufengine/models/moe.py:264-321) for mixed gate/up and down formats, and for the
routing edge cases: unused slots (-1), ids out of range, one expert chosen by every token, the
largest call (1024 pairs), token rows with a stride, run-to-run equality (the reference's
tests/test_moe.py:80)."""
import pytest
import torch
import torch.nn.functional as F

from nemicli_terminal_b200 import _lib, layers, moe, synth
from nemicli_terminal_b200.formats import FORMATS, TYPE_ID
from oracle import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu


def _experts(fmt, n_exp, n_out, n_in, seed, cuda):
    raw = synth.blocks(fmt, n_exp * n_out, n_in, seed=seed).view(n_exp, -1).to(cuda)
    return layers.PackedExperts(raw, TYPE_ID[fmt], n_exp, n_out, n_in, torch.bfloat16)


def _pair(gate, up, down):
    """(grouped MoeFFN, per-slot MoeFFN) over the same experts."""
    return moe.MoeFFN(gate, up, down), moe.MoeFFN(gate, up, down, act=lambda t: F.silu(t))


def _dense(fmt, raw_e, n_out, n_in):
    return torch.from_numpy(O.dequant(fmt, raw_e.cpu().numpy(), n_out * n_in)).view(n_out, n_in).double()


def _ref(fmts, ex, x, idx, w):
    """dense fp64: sum_j w * down(silu(gate x) * up x), slots with ids outside [0, n_exp) skipped."""
    gate, up, down = ex
    L, E = x.shape
    xc, ic, wc = x.cpu().double(), idx.cpu(), w.cpu().double()
    ref = torch.zeros(L, E, dtype=torch.float64)
    cache = {}

    def dense(i, e):
        if (i, e) not in cache:
            m = ex[i]
            cache[(i, e)] = _dense(fmts[i], m.raw[e], m.n_out, m.n_in)
        return cache[(i, e)]
    for t in range(L):
        for j in range(idx.shape[1]):
            e = int(ic[t, j])
            if not 0 <= e < gate.n_exp:
                continue
            a = F.silu(dense(0, e) @ xc[t]) * (dense(1, e) @ xc[t])
            ref[t] += wc[t, j] * (dense(2, e) @ a)
    return ref


def _rel(a, b):
    return O.max_rel(a.cpu().double().numpy(), b.cpu().double().numpy())


@pytest.mark.parametrize("fmt", H.FMTS)
def test_grouped_matches_per_slot(cuda, fmt):
    """Every format as gate, up and down: the grouped call agrees with the per-slot path."""
    n_exp, E, n_ff, L, k = 6, 512, 256, 5, 3
    gate, up, down = (_experts(fmt, n_exp, n_ff, E, 11, cuda), _experts(fmt, n_exp, n_ff, E, 12, cuda),
                      _experts(fmt, n_exp, E, n_ff, 13, cuda))
    grouped, per_slot = _pair(gate, up, down)
    x = synth.activations(L, E, seed=14, device=cuda)
    idx = torch.tensor([[0, 2, 5], [2, 0, 1], [5, 5, 3], [4, 2, 0], [1, 3, 2]], device=cuda)
    w = torch.rand(L, k, generator=torch.Generator().manual_seed(15)).to(cuda)
    out = grouped.grouped_call(x, idx, w)
    # both paths form silu(g) * u from the same sums; a last-bit difference in a value can move its
    # 8-bit code (a step of the group's maximum / 127 / 254 in the second stage), hence 1e-4
    assert _rel(out, per_slot(x, idx, w)) < 1e-4
    assert torch.equal(out, grouped(x, idx, w))


@pytest.mark.parametrize("L", [1, 3, 16])
def test_mixed_formats_dense(cuda, L):
    """Q4_K gate/up with Q6_K down (the common GGUF mix), bf16 input, against dense fp64."""
    n_exp, E, n_ff, k = 8, 1024, 512, 4
    fmts = ("Q4_K", "Q4_K", "Q6_K")
    ex = (_experts("Q4_K", n_exp, n_ff, E, 21, cuda), _experts("Q4_K", n_exp, n_ff, E, 22, cuda),
          _experts("Q6_K", n_exp, E, n_ff, 23, cuda))
    ffn = moe.MoeFFN(*ex)
    x = synth.activations(L, E, seed=24, device=cuda).to(torch.bfloat16)
    idx, w = moe.route(synth.router_logits(L, n_exp, seed=25, device=cuda), k)
    ref = _ref(fmts, ex, x.float(), idx, w)
    out = ffn.grouped_call(x, idx, w)
    assert _rel(out, ref) < 1e-3
    assert torch.equal(out, ffn.grouped_call(x, idx, w))
    assert _rel(ffn(x, idx, w), ref) < 1e-3             # whichever path __call__ takes at this size


def test_largest_call_and_fallback(cuda):
    """256 tokens x 4 slots (the grouped limit of 1024 pairs) with every token on expert 0 in slot 0
    (256 pairs of one expert, 64 passes of 4); 257 tokens are refused by the grouped call (and __call__
    takes the per-slot path)."""
    n_exp, E, n_ff, k = 16, 256, 128, 4
    ex = (_experts("Q8_0", n_exp, n_ff, E, 31, cuda), _experts("Q8_0", n_exp, n_ff, E, 32, cuda),
          _experts("Q4_0", n_exp, E, n_ff, 33, cuda))
    grouped, per_slot = _pair(*ex)
    for L in (256, 257):
        x = synth.activations(L, E, seed=34 + L, device=cuda)
        idx, w = moe.route(synth.router_logits(L, n_exp, seed=35 + L, device=cuda), k)
        idx[:, 0] = 0
        ref = per_slot(x, idx, w)
        if L == 256:
            out = grouped.grouped_call(x, idx, w)
            assert _rel(out, ref) < 1e-4
            assert torch.equal(out, grouped.grouped_call(x, idx, w))
        else:
            with pytest.raises(ValueError):
                grouped.grouped_call(x, idx, w)
            assert torch.equal(grouped(x, idx, w), ref)


def test_strided_rows(cuda):
    """Token rows further apart than dim (the expert-sharded exchange buffer: dim values, then the id
    columns) give the same result as the same rows packed."""
    n_exp, E, n_ff, L, k = 8, 512, 256, 6, 2
    ex = (_experts("Q4_K", n_exp, n_ff, E, 61, cuda), _experts("Q4_K", n_exp, n_ff, E, 62, cuda),
          _experts("Q6_K", n_exp, E, n_ff, 63, cuda))
    buf = torch.randn(L, E + 4, device=cuda)
    idx, w = moe.route(synth.router_logits(L, n_exp, seed=64, device=cuda), k)
    a = moe.grouped_ffn(*ex, buf[:, :E], idx, w)
    b = moe.grouped_ffn(*ex, buf[:, :E].contiguous(), idx, w)
    assert torch.equal(a, b)


def test_unused_and_refused_ids(cuda):
    """-1 (an unused slot) adds nothing and sets no status; an id outside [0, n_exp) adds nothing and
    sets the device status bit."""
    n_exp, E, n_ff, L, k = 4, 512, 256, 3, 2
    fmts = ("IQ2_XXS", "IQ2_XXS", "Q5_K")
    ex = (_experts("IQ2_XXS", n_exp, n_ff, E, 41, cuda), _experts("IQ2_XXS", n_exp, n_ff, E, 42, cuda),
          _experts("Q5_K", n_exp, E, n_ff, 43, cuda))
    ffn = moe.MoeFFN(*ex)
    x = synth.activations(L, E, seed=44, device=cuda)
    w = torch.full((L, k), 0.5, device=cuda)
    _lib.device_status(clear=True)
    idx = torch.tensor([[1, -1], [-1, -1], [3, 0]], device=cuda)
    out = ffn(x, idx, w)
    assert _lib.device_status(clear=True) == 0
    assert torch.count_nonzero(out[1]) == 0
    assert _rel(out, _ref(fmts, ex, x, idx, w)) < 1e-3
    bad = torch.tensor([[1, 7], [-1, -1], [3, 0]], device=cuda)
    assert torch.equal(ffn(x, bad, w), out)
    assert _lib.device_status(clear=True) & 1


def test_shapes_refused(cuda):
    """Inputs the grouped call cannot take raise instead of computing something else."""
    lib = _lib.load()
    assert lib.qmv_moe_workspace_bytes(0, 8, 2048, 768) == 0
    assert lib.qmv_moe_workspace_bytes(4, 8, 2048, 770) == 0
    n_exp, E, n_ff = 4, 512, 256
    ex = (_experts("Q4_K", n_exp, n_ff, E, 51, cuda), _experts("Q4_K", n_exp, n_ff, E, 52, cuda),
          _experts("Q4_K", n_exp, E, n_ff, 53, cuda))
    ffn = moe.MoeFFN(*ex, act=torch.tanh)
    x = synth.activations(2, E, seed=54, device=cuda)
    idx = torch.zeros(2, 2, dtype=torch.int64, device=cuda)
    with pytest.raises(ValueError):
        ffn.grouped_call(x, idx, torch.ones(2, 2, device=cuda))
    assert FORMATS["Q4_K"][0] == 256
