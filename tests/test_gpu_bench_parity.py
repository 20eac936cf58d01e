"""Parity of exactly what bench.py measures, at the benchmark's full sizes.

* the decode chain (`--mode chain`): the 32-layer, 128-stage Llama-3-8B projection stack that bench.py builds
  (bench.build_chain), captured in a CUDA graph and replayed several times; every stage's outputs are
  checked against the per-call API (mmvq.mv on the stage input recomputed in torch from the chain's own
  earlier outputs, 1e-5), and the stages of three layers against the dequantise-and-matmul oracle (oracle
  A, 1e-3);
* the per-call step (bench.build_calls, `--mode calls`, the BENCH value): replays identical, every output
  bit-identical to the unfused calls (norm_q8 / akt_q8 then the matvecs) on its own inputs, oracle A at
  three layers, with and without PDL;
* the batch-4 and batch-8 stack lines (bench.step_fn: the few-token tensor-core kernels) against the
  integer-path oracle (1e-5) and oracle A (1e-3);
* the config-4 MoE FFN (128 Q4_K experts, gate/up 768x2048, down 2048x768, top-8) at batch 1, 4 and 16
  against a dense fp64 computation with the dequantised experts (1e-3);
* mmvq.mm and QuantLinear at 17, 32 and 112 tokens (the reference's mm range) against both oracles.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import bench
from nemicli_terminal_b200 import chain, layers, mmvq, moe, qlinear, synth
from nemicli_terminal_b200.formats import TYPE_ID
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = torch.as_tensor(a).double().cpu(), torch.as_tensor(b).double().cpu()
    return float((a - b).abs().max() / b.abs().max().clamp_min(1e-30))


def _dense(fmt, raw, n_out, n_in):
    """Oracle A's weights: the dequantised matrix (bit-identical with the reference's dequantize), fp64."""
    return torch.from_numpy(O.dequant(fmt, raw.reshape(-1).cpu().numpy(), n_out * n_in)).view(n_out, n_in).double()


def _rmsnorm(v, w, eps):
    return v * torch.rsqrt(v.pow(2).mean() + eps) * w


@pytest.fixture(scope="module")
def stack(cuda):
    return bench.build_stack(cuda, seed0=0)


def test_headline_chain_128_stages(cuda, stack):
    """bench.py's chain (the BENCH value): graph replays are identical; every stage matches the per-call
    path; layers 0, 15 and 31 match oracle A."""
    ch, h0, last, outs = bench.build_chain(stack, cuda, seed=0)
    assert len(ch.stages) == 4 * bench.LAYERS == 128
    g, _ = bench.capture(lambda: ch.run())
    snaps = []
    for _ in range(3):
        for st in ch.stages:                 # poison the outputs: each replay must rewrite all of them
            for y in st.ys:
                y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        snaps.append([y.clone() for st in ch.stages for y in st.ys])
    for s in snaps[1:]:
        assert all(torch.equal(a, b) for a, b in zip(snaps[0], s))
    eps = 1e-5
    h, r = h0, None
    for l in range(bench.LAYERS):
        s1, s2, s3, s4 = ch.stages[4 * l:4 * l + 4]
        m = {name: (fmt, raw, n_out, n_in) for name, fmt, n_out, n_in, slot, raw in stack[l]}
        hin = h if r is None else h + r
        x1 = _rmsnorm(hin, s1.norm_w, eps)
        for name, y in zip(("q", "k", "v"), s1.ys):
            f, raw, n_out, n_in = m[name]
            assert _rel(y, mmvq.mv(f, raw, x1, n_out, n_in)) < 1e-5, (l, name)
        f, raw, n_out, n_in = m["o"]
        assert _rel(s2.ys[0], mmvq.mv(f, raw, s1.ys[0], n_out, n_in)) < 1e-5, (l, "o")
        hm = hin + s2.ys[0]
        assert torch.equal(s3.h_out, hm), l
        x3 = _rmsnorm(hm, s3.norm_w, eps)
        for name, y in zip(("gate", "up"), s3.ys):
            f, raw, n_out, n_in = m[name]
            assert _rel(y, mmvq.mv(f, raw, x3, n_out, n_in)) < 1e-5, (l, name)
        x4 = F.silu(s3.ys[0]) * s3.ys[1]
        f, raw, n_out, n_in = m["down"]
        assert _rel(s4.ys[0], mmvq.mv(f, raw, x4, n_out, n_in)) < 1e-5, (l, "down")
        if l in (0, 15, 31):
            # oracle A from the same stage inputs, in fp64 (no quantised activation)
            for name, x, y in (("q", x1, s1.ys[0]), ("k", x1, s1.ys[1]), ("v", x1, s1.ys[2]),
                               ("o", s1.ys[0], s2.ys[0]), ("gate", x3, s3.ys[0]), ("up", x3, s3.ys[1]),
                               ("down", x4, s4.ys[0])):
                f, raw, n_out, n_in = m[name]
                ya = _dense(f, raw, n_out, n_in) @ x.double().cpu()
                assert _rel(y, ya) < 1e-3, (l, name)
        h, r = hm, s4.ys[0]
    assert last.data_ptr() == ch.stages[-1].ys[0].data_ptr()


@pytest.mark.parametrize("pdl", [False, True])
def test_headline_calls_128_stages(cuda, stack, pdl):
    """bench.py's per-call step (--mode calls), with PDL (the bench: separate producer launches that
    overlap) and without (norms and quantisation inside the matvecs): graph replays are identical; every
    output equals, bit for bit, the unfused calls (norm_q8, then the matvecs on its Eingang; akt_q8, then
    down) fed with the step's own earlier outputs; layers 0, 15 and 31 match oracle A; layer 0 matches
    the chain."""
    old = mmvq.pdl(pdl)
    try:
        _calls_step_parity(cuda, stack)
    finally:
        mmvq.pdl(old)


def _calls_step_parity(cuda, stack):
    step, h0, last = bench.build_calls(stack, cuda, seed=0)
    g, outs = bench.capture(step)
    assert len(outs) == 7 * bench.LAYERS
    snaps = []
    for _ in range(3):
        for y in outs:
            y.fill_(float("nan"))
        g.replay()
        torch.cuda.synchronize()
        snaps.append([y.clone() for y in outs])
    for s in snaps[1:]:
        assert all(torch.equal(a, b) for a, b in zip(snaps[0], s))
    eps = 1e-5
    h, r = h0, None
    for l in range(bench.LAYERS):
        q, k, v, o, gt, up, d = outs[7 * l:7 * l + 7]
        wa, wf = step.norms[l]
        m = {name: (fmt, raw, n_out, n_in) for name, fmt, n_out, n_in, slot, raw in stack[l]}
        x1, e1, h = mmvq.norm_q8(h, wa, eps, r)
        ref = mmvq.mv_geteilt("Q4_K", [(m[x][1], m[x][2]) for x in ("q", "k", "v")], e1, 4096)
        assert all(torch.equal(a, b) for a, b in zip((q, k, v), ref)), l
        assert torch.equal(o, mmvq.mv("Q4_K", m["o"][1], mmvq.Eingang(q), 4096, 4096)), l
        x3, e3, h = mmvq.norm_q8(h, wf, eps, o)
        ref = mmvq.mv_geteilt("Q4_K", [(m[x][1], m[x][2]) for x in ("gate", "up")], e3, 4096)
        assert all(torch.equal(a, b) for a, b in zip((gt, up), ref)), l
        x4, e4 = mmvq.akt_q8(gt, up, False)
        assert torch.equal(d, mmvq.mv("Q6_K", m["down"][1], e4, 4096, 14336)), l
        if l in (0, 15, 31):
            for name, x, y in (("q", x1, q), ("k", x1, k), ("v", x1, v), ("o", q, o), ("gate", x3, gt),
                               ("up", x3, up), ("down", x4, d)):
                f, raw, n_out, n_in = m[name]
                ya = _dense(f, raw, n_out, n_in) @ x.double().cpu()
                assert _rel(y, ya) < 1e-3, (l, name)
        r = d
    assert last[0].data_ptr() == outs[-1].data_ptr()
    ch, _, _, chain_outs = bench.build_chain(stack[:1], cuda, seed=0)
    ch.run()
    torch.cuda.synchronize()
    for a, b in zip(chain_outs, snaps[0][:7]):
        assert _rel(a, b) < 1e-4


@pytest.mark.parametrize("batch", [4, 8])
def test_stack_batches(cuda, stack, batch):
    """bench.step_fn at batch 4 / 8 (the BENCH `batches` lines) on two layers of the stack."""
    two = stack[:2]
    xs = [[synth.activations(batch, n, seed=7919 * l + s + batch, device=cuda) for s, n in enumerate(bench.INPUTS)]
          for l in range(2)]
    outs = bench.step_fn(two, xs, batch)
    i = 0
    for l, mats in enumerate(two):
        for slot in range(4):
            for name, fmt, n_out, n_in, s_, raw in [mm for mm in mats if mm[4] == slot]:
                y = outs[i]
                i += 1
                x = xs[l][slot].cpu()
                qa = O.quant_q8(x.numpy().reshape(-1))
                yb = O.mv(fmt, raw.cpu().numpy(), n_out, n_in, *qa, n_tok=batch)
                assert O.max_rel(y.cpu().numpy(), yb) < 1e-5, (l, name)
                ya = (_dense(fmt, raw, n_out, n_in) @ x.double().t()).t()
                assert _rel(y, ya) < 1e-3, (l, name)
    assert i == len(outs)


def _experts(n_exp, n_out, n_in, seed, device):
    return synth.blocks("Q4_K", n_exp * n_out, n_in, seed=seed, device=device)


@pytest.fixture(scope="module")
def moe_cfg4(cuda):
    E, n_ff, n_exp = bench.MOE_DIM, bench.MOE_FF, bench.MOE_EXPERTS
    mk = lambda n_out, n_in, seed: layers.PackedExperts(_experts(n_exp, n_out, n_in, seed, cuda), TYPE_ID["Q4_K"],  # noqa: E731
                                                        n_exp, n_out, n_in, torch.float32)
    return mk(n_ff, E, 700), mk(n_ff, E, 701), mk(E, n_ff, 702)


@pytest.mark.parametrize("L", [1, 4, 16])
def test_moe_config4(cuda, moe_cfg4, L):
    gate, up, down = moe_cfg4
    E, n_ff, k = bench.MOE_DIM, bench.MOE_FF, bench.MOE_K
    ffn = moe.MoeFFN(gate, up, down)
    x = synth.activations(L, E, seed=710 + L, device=cuda)
    idx, w = moe.route(synth.router_logits(L, bench.MOE_EXPERTS, seed=720 + L, device=cuda), k)
    out = ffn(x, idx, w)
    xc, ic, wc = x.cpu().double(), idx.cpu(), w.cpu().double()
    cache = {}

    def dense(ex, e, n_out, n_in):
        key = (id(ex), e)
        if key not in cache:
            cache[key] = _dense("Q4_K", ex.raw[e], n_out, n_in)
        return cache[key]
    ref = torch.zeros(L, E, dtype=torch.float64)
    for t in range(L):
        for j in range(k):
            e = int(ic[t, j])
            a = F.silu(dense(gate, e, n_ff, E) @ xc[t]) * (dense(up, e, n_ff, E) @ xc[t])
            ref[t] += wc[t, j] * (dense(down, e, E, n_ff) @ a)
    assert _rel(out, ref) < 1e-3
    assert torch.equal(out, ffn(x, idx, w))


@pytest.mark.parametrize("fmt,n_out,n_in", [("Q4_K", 4096, 4096), ("Q6_K", 1024, 14336), ("Q8_0", 2048, 4096),
                                            ("IQ2_XXS", 1024, 4096)])
@pytest.mark.parametrize("M", [17, 32, 112])
def test_mm_long_inputs(cuda, fmt, n_out, n_in, M):
    raw = synth.blocks(fmt, n_out, n_in, seed=M, device=cuda)
    x = synth.activations(M, n_in, seed=M + 1, device=cuda)
    y = mmvq.mm(fmt, raw, x, n_out, n_in)
    assert y.shape == (M, n_out)
    xc = x.cpu()
    if mmvq.tc_used(fmt, M, n_out, n_in):  # the tensor-core tile path: the reference MMQ's fp16 arithmetic
        yc = O.mmq(fmt, raw.cpu().numpy(), n_out, n_in, xc.numpy())
        assert O.max_rel(y.cpu().numpy(), yc) < 2e-5
    else:
        qa = O.quant_q8(xc.numpy().reshape(-1))
        yb = O.mv(fmt, raw.cpu().numpy(), n_out, n_in, *qa, n_tok=M)
        assert O.max_rel(y.cpu().numpy(), yb) < 1e-5
    ya = (_dense(fmt, raw, n_out, n_in) @ xc.double().t()).t()
    assert _rel(y, ya) < 1e-3


@pytest.mark.parametrize("fmt", ["Q4_0", "Q8_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("M", [17, 32, 112])
def test_quant_linear_long_inputs(cuda, fmt, M):
    n_out, n_in = 1024, 4096
    raw = synth.blocks(fmt, n_out, n_in, seed=3 * M, device=cuda)
    ql = qlinear.build_quant_linear(raw, TYPE_ID[fmt], n_out, n_in)
    x = synth.activations(M, n_in, seed=M, device=cuda).to(torch.bfloat16)
    y = ql(x)
    assert y.dtype == torch.bfloat16 and y.shape == (M, n_out)
    ya = (_dense(fmt, raw, n_out, n_in) @ x.cpu().double().t()).t()
    assert _rel(y.float(), ya) < 1e-2            # bf16 output rounding (the reference's QuantLinear returns bf16)
    yf = mmvq.mm(fmt, raw, x, n_out, n_in)
    assert _rel(yf, ya) < 1e-3
