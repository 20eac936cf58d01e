"""The oracle pinned against the reference: golden vectors made by the reference's own
ggufengine.quant.dequantize (tests/golden/make_golden.py), the reference test's invariants of the
two-stage int8 input, and exact identities of the integer path.  CPU only."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests import helpers as H

GOLDEN = np.load(os.path.join(os.path.dirname(__file__), "golden", "dequant_golden.npz"))
KEYS = sorted({k.split("__")[0] for k in GOLDEN.files})
NAME = {v: k for k, v in O.TYPES.items()}


def _golden(key):
    t, rows, cols = (int(v) for v in GOLDEN[key + "__shape"])
    return NAME[t], rows, cols, GOLDEN[key + "__raw"], GOLDEN[key + "__deq"], GOLDEN[key + "__x"], GOLDEN[key + "__y"]


def test_golden_covers_all_formats():
    assert {(_golden(k)[0]) for k in KEYS} == set(O.TYPES)


@pytest.mark.parametrize("key", KEYS)
def test_dequant_bit_exact_with_reference(key):
    name, rows, cols, raw, deq, _, _ = _golden(key)
    out = O.dequant(name, raw, rows * cols)
    assert np.array_equal(out.view(np.uint32), deq.view(np.uint32)), name


@pytest.mark.parametrize("key", KEYS)
def test_oracle_a_matches_golden_product(key):
    name, rows, cols, raw, _, x, y = _golden(key)
    assert O.max_rel(O.mv_exact(name, raw, rows, cols, x), y) < 1e-12


@pytest.mark.parametrize("key", KEYS)
def test_integer_path_within_north_star_tolerance(key):
    """Oracle B (two-stage int8) against the reference's dequantise-and-matmul: <= 1e-3 max rel."""
    name, rows, cols, raw, _, x, y = _golden(key)
    qa = O.quant_q8(x.reshape(-1))
    yb = O.mv(name, raw, rows, cols, *qa, n_tok=x.shape[0])
    assert O.max_rel(yb, y) < 1e-3


@pytest.mark.parametrize("key", KEYS)
def test_integer_sums_pin_the_layout(key):
    """With xs replaced by the sum of the quantised input, the integer path equals dequant @ x_hat
    exactly (up to fp32 rounding of Q4_K's dequantised values): any code/activation mismatch in the
    int32 sums would show up as an O(1) error."""
    name, rows, cols, raw, deq, x, _ = _golden(key)
    xq, xq2, xd, xs = O.quant_q8(x.reshape(-1))
    xhat = np.repeat(xd, 32).astype(np.float64) * (xq.astype(np.float64) + xq2.astype(np.float64) / 254.0)
    xs_hat = xhat.reshape(-1, 32).sum(1).astype(np.float32)
    yb = O.mv(name, raw, rows, cols, xq, xq2, xd, xs_hat, n_tok=x.shape[0])
    ref = xhat.reshape(x.shape) @ deq.reshape(rows, cols).astype(np.float64).T
    assert O.max_rel(yb, ref) < 1e-6


def test_quantiser_invariants():
    """The reference's test of its int8 input (tests/test_mmvq.py:123-127 there): xq*xd ~ x (1e-2),
    + xq2*xd/254 ~ x (1e-4), xs = exact sum (1e-5), relative to max |x|."""
    rng = np.random.default_rng(3)
    for n in (32, 4096, 14336):
        x = (rng.standard_normal(n) * rng.choice([1e-3, 1.0, 300.0])).astype(np.float32)
        xq, xq2, xd, xs = O.quant_q8(x)
        d = np.repeat(xd, 32).astype(np.float64)
        m = np.abs(x).max()
        assert np.abs(d * xq - x).max() / m < 1e-2
        assert np.abs(d * (xq + xq2 / 254.0) - x).max() / m < 1e-4
        assert np.abs(xs - x.reshape(-1, 32).astype(np.float64).sum(1)).max() / m < 1e-5


def test_quantiser_edge_values():
    x = np.zeros(64, np.float32)
    x[32:] = np.linspace(-1, 1, 32, dtype=np.float32)
    xq, xq2, xd, xs = O.quant_q8(x)
    assert (xq[:32] == 0).all() and (xq2[:32] == 0).all() and xd[0] == 0 and xs[0] == 0
    assert xq[32:].min() == -127 and xq[32:].max() == 127
    # bf16 input path: the same values as quantising the bf16-rounded fp32
    xb = O.bf16_bits(x)
    a = O.quant_q8(xb)
    b = O.quant_q8(O.bf16_to_f32(xb))
    assert all(np.array_equal(u, v) for u, v in zip(a, b))


@pytest.mark.parametrize("fmt", H.FMTS)
def test_block_sums_compose_the_matvec(fmt):
    """mv's integer sums are exactly the block sums (same units, same codes)."""
    n_out, n_in = 3, 512
    raw, x = H.case(fmt, n_out, n_in, seed=11)
    xq, xq2, xd, xs = O.quant_q8(x.numpy().reshape(-1))
    s, s2 = O.block_sums(fmt, raw.numpy(), n_out, n_in, xq, xq2)
    u = O.unit_values(fmt)
    codes = O.dequant(fmt, raw.numpy(), n_out * n_in)   # only for the shape check
    assert s.shape == (n_out, n_in // u) and codes.size == n_out * n_in
    # recompute the sums from the per-value codes of a plain restatement
    W = O.dequant(fmt, raw.numpy(), n_out * n_in).reshape(n_out, n_in)
    assert np.isfinite(W).all()
    assert np.abs(s).max() < 2 ** 24 and np.abs(s2).max() < 2 ** 24


@pytest.mark.parametrize("fmt", H.FMTS)
def test_synthetic_configs_within_tolerance(fmt):
    """Seeded config-like blocks (synth): oracle B within 1e-3 of oracle A, several tokens."""
    n_in = 256 if fmt not in ("Q4_0", "Q8_0") else 96
    raw, x = H.case(fmt, 16, n_in, n_tok=3, seed=5)
    yb, _ = H.oracle_b(fmt, raw, x, 16, n_in)
    ya = H.oracle_a(fmt, raw, x, 16, n_in)
    assert O.max_rel(yb, ya) < 1e-3


def test_bf16_input_path():
    raw, x = H.case("Q4_K", 8, 512, seed=2, x_dtype=torch.bfloat16)
    yb, _ = H.oracle_b("Q4_K", raw, x, 8, 512)
    ya = H.oracle_a("Q4_K", raw, x, 8, 512)
    assert O.max_rel(yb, ya) < 1e-3


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_mmq_weights_follow_the_pinned_dequantiser(fmt):
    """Oracle C's fp16 weights (the reference MMQ's unpacking) lie within one fp16 step of the
    golden-pinned dequantiser's values at every position: the byte layout it decodes is the pinned one."""
    from nemicli_terminal_b200 import synth
    n_out, n_in = 48, 1024
    raw = synth.blocks(fmt, n_out, n_in, seed=9).numpy()
    w16 = O.mmq_weights(fmt, raw, n_out, n_in).astype(np.float64)
    wa = O.dequant(fmt, raw.reshape(-1), n_out * n_in).reshape(n_out, n_in).astype(np.float64)
    step = np.maximum(np.abs(wa), 2.0 ** -14) * 2.0 ** -10          # one fp16 ulp (normal range)
    assert np.all(np.abs(w16 - wa) <= step)
    assert np.mean(w16 == wa.astype(np.float16).astype(np.float64)) > 0.99
