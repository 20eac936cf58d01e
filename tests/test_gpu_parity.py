"""Parity of the CUDA path with the oracle (GPU).

* the activation quantiser is bit-exact with the oracle's restatement,
* the int32 unit sums of every format are bit-exact with the oracle (same activation input),
* fp32 outputs are within 1e-5 max-rel of the integer-path oracle (fp64 epilogue) and within the
  north-star 1e-3 max-rel of the reference's dequantise-and-matmul (oracle A),
at the reference tests' shapes (tests/test_mmvq.py:57 there: (256, 512), (1024, 4096), (300, 1280)),
the golden fixtures, and the benchmark configs' full sizes through sampled rows and exact scaling.
"""
import os

import numpy as np
import pytest
import torch

from nemicli_terminal_b200 import mmvq, synth
from nemicli_terminal_b200.formats import FORMATS, row_bytes
from oracle import oracle as O
from tests import helpers as H

pytestmark = pytest.mark.gpu

TOL_B = 1e-5      # GPU fp32 epilogue vs oracle B (exact int sums, fp64 epilogue)
TOL_A = 1e-3      # north star: vs the reference's dequantise-and-matmul

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "dequant_golden.npz"))
GKEYS = sorted({k.split("__")[0] for k in GOLDEN.files})
NAME = {v: k for k, v in O.TYPES.items()}


def _shapes(fmt):
    bv = FORMATS[fmt][0]
    if bv == 32:
        return [(256, 512), (1024, 4096), (300, 1280), (7, 96), (33, 32)]
    return [(256, 512), (1024, 4096), (300, 1280), (5, 256), (300, 2048)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [32, 4096, 14336, 32 * 999])
def test_quantiser_bit_exact(cuda, dtype, n):
    x = synth.activations(1, n, seed=n).to(dtype).reshape(-1)
    x[:32] = 0                                       # an all-zero group
    x[32:64] *= 1e-30                                # tiny values (subnormal scales)
    e = mmvq.Eingang(x.to(cuda))
    ref = O.quant_q8(H.x_numpy(x))
    got = [e.xq.cpu().numpy(), e.xq2.cpu().numpy(), e.xd.cpu().numpy(), e.xs.cpu().numpy()]
    for g, r in zip(got, ref):
        assert np.array_equal(g.view(np.uint8) if g.dtype == np.int8 else g.view(np.uint32),
                              r.view(np.uint8) if r.dtype == np.int8 else r.view(np.uint32))


@pytest.mark.parametrize("fmt", H.FMTS)
def test_block_sums_bit_exact(cuda, fmt):
    for n_out, n_in in _shapes(fmt):
        raw, x = H.case(fmt, n_out, n_in, seed=n_out)
        e = mmvq.Eingang(x.to(cuda))
        s, s2 = mmvq.block_sums(fmt, raw.to(cuda), e, n_out, n_in)
        rs, rs2 = O.block_sums(fmt, raw.numpy(), n_out, n_in, e.xq.cpu().numpy(), e.xq2.cpu().numpy())
        assert np.array_equal(s.cpu().numpy(), rs), (fmt, n_out, n_in)
        assert np.array_equal(s2.cpu().numpy(), rs2), (fmt, n_out, n_in)


@pytest.mark.parametrize("fmt", H.FMTS)
@pytest.mark.parametrize("n_tok", [1, 2, 3, 4, 5, 8, 9, 16])
def test_mv_matches_oracles(cuda, fmt, n_tok):
    for n_out, n_in in _shapes(fmt):
        raw, x = H.case(fmt, n_out, n_in, n_tok=n_tok, seed=n_out + n_tok)
        y = mmvq.mv(fmt, raw.to(cuda), x.to(cuda), n_out, n_in).cpu().numpy()
        yb, _ = H.oracle_b(fmt, raw, x, n_out, n_in)
        ya = H.oracle_a(fmt, raw, x, n_out, n_in)
        assert y.shape == (n_tok, n_out)
        assert O.max_rel(y, yb) < TOL_B, (fmt, n_out, n_in, n_tok)
        assert O.max_rel(y, ya) < TOL_A, (fmt, n_out, n_in, n_tok)


@pytest.mark.parametrize("fmt", H.FMTS)
def test_input_forms_agree(cuda, fmt):
    """x as fp32, as bf16, and as a prepared Eingang (the reference's three forms, test_mmvq.py:61)."""
    n_out, n_in = 64, 1024
    raw, x = H.case(fmt, n_out, n_in, seed=3)
    r = raw.to(cuda)
    xc = x[0].to(cuda)
    y32 = mmvq.mv(fmt, r, xc, n_out, n_in)
    ye = mmvq.mv(fmt, r, mmvq.Eingang(xc), n_out, n_in)
    assert y32.shape == (n_out,) and ye.shape == (n_out,)
    assert torch.equal(y32, ye)
    yb16 = mmvq.mv(fmt, r, xc.to(torch.bfloat16), n_out, n_in).cpu().numpy()
    yb, _ = H.oracle_b(fmt, raw, x.to(torch.bfloat16), n_out, n_in)
    assert O.max_rel(yb16, yb[0]) < TOL_B


@pytest.mark.parametrize("fmt,n_in", [("Q8_0", 256), ("Q8_0", 4352), ("Q4_0", 14336 + 256), ("Q4_K", 14336),
                                       ("IQ2_XXS", 14336), ("TQ2_0", 10240)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_quantisation_equals_eingang(cuda, fmt, n_in, dtype):
    """The one-token kernel quantises the row itself, a group on each eighth of a warp (the last round
    of a warp partly past the row's end): bit-identical to the separate quantiser's input.  Rows past
    FUSED_MAX_IN are forced onto the fused kernel (mv takes the separate quantiser there)."""
    n_out = 512
    raw = synth.blocks(fmt, n_out, n_in, seed=n_in, device=cuda)
    x = synth.activations(1, n_in, seed=5, device=cuda)[0].to(dtype)
    fused = mmvq._fused(fmt, [(raw, n_out)], x, n_in, force=True)
    assert fused is not None                      # rows of a multiple of 16 bytes: the staged kernel
    fused = fused[0]
    assert torch.equal(fused, mmvq.mv(fmt, raw, mmvq.Eingang(x), n_out, n_in))
    assert torch.equal(mmvq.mv(fmt, raw, x, n_out, n_in), fused)


def test_fused_quantisation_ties(cuda):
    """Values exactly on the half-way points of the 8-bit steps (group maximum 15.875, so the step d
    is 1/8 and v = (k + 1/2) / 8 divides to a tie), their fp32 neighbours, the steps themselves, all-zero
    groups and groups with one nonzero value: the fused kernel's input equals the separate quantiser's."""
    n_in, n_out = 4096, 256
    k = torch.arange(-127, 127, dtype=torch.float32)
    half = (k + 0.5) / 8
    vals = torch.cat([half, torch.nextafter(half, torch.tensor(16.0)), torch.nextafter(half, torch.tensor(-16.0)),
                      k / 8])
    x = torch.zeros(n_in)
    n_full = (vals.numel() + 30) // 31
    for g in range(n_full):
        part = vals[31 * g: 31 * g + 31]
        x[32 * g: 32 * g + part.numel()] = part
        x[32 * g + 31] = 15.875 if g % 2 else -15.875
    for g in range(n_full + 8, n_in // 32, 2):               # one nonzero value; the others stay zero groups
        x[32 * g + g % 32] = 1e-3 * (g - 60)
    xc = x.to(cuda)
    raw = synth.blocks("Q8_0", n_out, n_in, seed=9, device=cuda)
    e = mmvq.Eingang(xc)
    assert int((e.xd[:n_full].cpu() == 0.125).sum()) == n_full
    fused = mmvq._fused("Q8_0", [(raw, n_out)], xc, n_in, force=True)[0]
    assert torch.equal(fused, mmvq.mv("Q8_0", raw, e, n_out, n_in))


@pytest.mark.parametrize("fmt", ["Q4_K", "Q8_0", "Q6_K", "IQ2_XXS"])
@pytest.mark.parametrize("n_tok", [1, 2, 5, 8, 11])
def test_several_matrices_equal_single_calls(cuda, fmt, n_tok):
    """mv_geteilt on several matrices (three, of 512, 136 and 256 rows, sharing one input) gives, bit for
    bit, what one mv per matrix gives: at several tokens Q4_K and Q8_0 run all matrices in one
    tensor-core launch (one tile list over the matrices; the 136-row matrix ends in a half tile)."""
    n_in = 4096
    mats = [(synth.blocks(fmt, n_out, n_in, seed=n_out + n_tok, device=cuda), n_out) for n_out in (512, 136, 256)]
    e = mmvq.Eingang(synth.activations(n_tok, n_in, seed=n_tok, device=cuda))
    ys = mmvq.mv_geteilt(fmt, mats, e, n_in)
    for (raw, n_out), y in zip(mats, ys):
        ref = mmvq.mv(fmt, raw, e, n_out, n_in)
        assert y.shape == ref.shape
        assert torch.equal(y, ref)


@pytest.mark.parametrize("key", GKEYS)
def test_golden_fixtures_on_gpu(cuda, key):
    t, rows, cols = (int(v) for v in GOLDEN[key + "__shape"])
    fmt = NAME[t]
    raw = torch.from_numpy(GOLDEN[key + "__raw"].copy())
    x = torch.from_numpy(GOLDEN[key + "__x"].copy())
    y = mmvq.mv(fmt, raw.to(cuda), x.to(cuda), rows, cols).cpu().numpy()
    assert O.max_rel(y, GOLDEN[key + "__y"]) < TOL_A


def test_run_to_run_deterministic(cuda):
    raw, x = H.case("Q4_K", 4096, 4096, n_tok=4, seed=1)
    r, xc = raw.to(cuda), x.to(cuda)
    a = mmvq.mv("Q4_K", r, xc, 4096, 4096)
    b = mmvq.mv("Q4_K", r, xc, 4096, 4096)
    assert torch.equal(a, b)


# benchmark configs at full size: sampled rows against the oracle, and exact power-of-two scaling
CONFIGS = [
    ("Q4_0", 4096, 4096, (1,)),            # config 1
    ("Q4_K", 4096, 4096, (1, 4, 8)),       # config 2: q/o
    ("Q4_K", 1024, 4096, (1,)),            #           k/v
    ("Q4_K", 14336, 4096, (1, 8)),         #           gate/up
    ("Q6_K", 4096, 14336, (1, 4, 8)),      #           down
    ("Q8_0", 128256, 4096, (1, 8)),        # config 3
    ("Q6_K", 128256, 4096, (1,)),
    ("TQ2_0", 14336, 4096, (1,)),          # config 5
    ("TQ2_0", 4096, 14336, (1,)),
    ("IQ2_XXS", 14336, 4096, (1,)),
    ("IQ2_XXS", 4096, 14336, (1,)),
]


@pytest.mark.parametrize("fmt,n_out,n_in,toks", CONFIGS)
def test_full_size_configs(cuda, fmt, n_out, n_in, toks):
    raw = synth.blocks(fmt, n_out, n_in, seed=7, device=cuda)
    rb = row_bytes(fmt, n_in)
    rows = torch.unique(torch.cat([torch.tensor([0, n_out - 1]), torch.randint(0, n_out, (254,))])).tolist()
    sub = raw.view(n_out, rb)[rows].cpu()
    for T in toks:
        x = synth.activations(T, n_in, seed=T, device=cuda)
        y = mmvq.mv(fmt, raw, x, n_out, n_in)
        assert torch.isfinite(y).all()
        ys = y[:, rows].cpu().numpy()
        xs = x.cpu()
        yb, _ = H.oracle_b(fmt, sub.reshape(-1), xs, len(rows), n_in)
        ya = H.oracle_a(fmt, sub.reshape(-1), xs, len(rows), n_in)
        assert O.max_rel(ys, yb) < TOL_B, (fmt, n_out, n_in, T)
        assert O.max_rel(ys, ya) < TOL_A, (fmt, n_out, n_in, T)
        # scaling the input by 2^k scales xd and xs exactly: the output scales bit for bit
        y4 = mmvq.mv(fmt, raw, x * 4.0, n_out, n_in)
        assert torch.equal(y4, y * 4.0)
