"""Decode chain (qmv_chain) against the per-call API on the GPU: every stage's input computed in torch
(RMS norm with the residual, SiLU gate), quantised and multiplied through mmvq.mv, compared with the
chain's outputs; plus the written residual streams and graph replay."""
import pytest
import torch
import torch.nn.functional as F

from nemicli_terminal_b200 import chain, mmvq, synth

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30))


def _layer(dev, seed, down_fmt="Q6_K"):
    mk = lambda fmt, n_out, n_in, s: (fmt, synth.blocks(fmt, n_out, n_in, seed=seed + s, device=dev), n_out, n_in)  # noqa: E731
    return (mk("Q4_K", 4096, 4096, 1), mk("Q4_K", 1024, 4096, 2), mk("Q4_K", 1024, 4096, 3), mk("Q4_K", 4096, 4096, 4),
            mk("Q4_K", 14336, 4096, 5), mk("Q4_K", 14336, 4096, 6), mk(down_fmt, 4096, 14336, 7))


def _rmsnorm(v, w, eps):
    return v * torch.rsqrt(v.pow(2).mean() + eps) * w


@pytest.mark.parametrize("down_fmt", ["Q6_K", "Q4_K"])
def test_two_layer_chain_matches_per_call(cuda, down_fmt):
    torch.manual_seed(0)
    eps = 1e-5
    layers = [_layer(cuda, 100 * i, down_fmt) for i in range(2)]
    norms = [(torch.rand(4096, device=cuda) + 0.5, torch.rand(4096, device=cuda) + 0.5) for _ in range(2)]
    h0 = synth.activations(1, 4096, seed=9, device=cuda)[0]
    stages, h, r = [], h0, None
    outs = []
    for i, (L, (wa, wf)) in enumerate(zip(layers, norms)):
        st, h_mid, y_down = chain.layer_stages(*L, h_in=h, resid_in=r, attn_norm=wa, ffn_norm=wf, eps=eps, first=i == 0)
        stages += st
        outs.append((st, h_mid, y_down))
        h, r = h_mid, y_down
    ch = chain.Chain(stages)
    ch.run()
    torch.cuda.synchronize()
    # per-call reference, stage by stage, from the chain's own earlier outputs
    h, r = h0, None
    for (st, h_mid, y_down), L, (wa, wf) in zip(outs, layers, norms):
        q, k, v, o, gate, up, down = L
        hin = h if r is None else h + r
        if r is not None:
            assert torch.equal(st[0].h_out, hin)
        x1 = _rmsnorm(hin, wa, eps)
        for m, y in zip((q, k, v), st[0].ys):
            assert _rel(y, mmvq.mv(m[0], m[1], x1, m[2], m[3])) < 1e-5
        assert _rel(st[1].ys[0], mmvq.mv(o[0], o[1], st[0].ys[0], o[2], o[3])) < 1e-5
        hm = hin + st[1].ys[0]
        assert torch.equal(h_mid, hm)
        x3 = _rmsnorm(hm, wf, eps)
        for m, y in zip((gate, up), st[2].ys):
            assert _rel(y, mmvq.mv(m[0], m[1], x3, m[2], m[3])) < 1e-5
        x4 = F.silu(st[2].ys[0]) * st[2].ys[1]
        assert _rel(y_down, mmvq.mv(down[0], down[1], x4, down[2], down[3])) < 1e-5
        h, r = h_mid, y_down


def test_chain_graph_replay_is_deterministic(cuda):
    L = _layer(cuda, 7)
    wa, wf = torch.ones(4096, device=cuda), torch.ones(4096, device=cuda)
    h0 = synth.activations(1, 4096, seed=3, device=cuda)[0]
    st, h_mid, y_down = chain.layer_stages(*L, h_in=h0, resid_in=None, attn_norm=wa, ffn_norm=wf, first=True)
    ch = chain.Chain(st)
    ch.run()
    torch.cuda.synchronize()
    ref = y_down.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ch.run()
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        ch.run()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_down, ref)


def test_chain_refuses_unsupported_shapes(cuda):
    raw = synth.blocks("Q4_K", 64, 2048, seed=1, device=cuda)
    x = torch.randn(2048, device=cuda)
    with pytest.raises(RuntimeError):
        chain.Chain([chain.Stage("Q4_K", [(raw, 64)], 2048, chain.RAW, a=x, wait=False)]).run()
