"""Host-side logic of the drop-in modules that needs no GPU: refusals without a CPU fallback,
dispatch tables, routing and the synthetic generators."""
import numpy as np
import pytest
import torch

from nemicli_terminal_b200 import cudakern, layers, mmvq, moe, qlinear, synth
from nemicli_terminal_b200.formats import FORMATS, GGML_TYPES, TYPE_ID, row_bytes
from oracle import oracle as O


def test_format_table_matches_ggml_types():
    for name, (bv, bb) in FORMATS.items():
        assert GGML_TYPES[TYPE_ID[name]] == (name, bv, bb)


def test_no_cpu_fallback():
    raw = synth.blocks("Q4_K", 4, 256)
    x = torch.randn(256)
    assert not mmvq.verfuegbar("cpu", "Q4_K", 256)
    assert not cudakern.verfuegbar("cpu", "Q4_K", 256)
    with pytest.raises(RuntimeError):
        mmvq.mv("Q4_K", raw, x, 4, 256)
    with pytest.raises(RuntimeError):
        mmvq.Eingang(x)
    with pytest.raises(RuntimeError):
        cudakern.mv("Q4_K", raw.view(1, -1), torch.zeros(1, dtype=torch.long), x, 4, 256)
    with pytest.raises(RuntimeError):
        layers.PackedLinear(raw, TYPE_ID["Q4_K"], 4, 256, None, torch.bfloat16)
    with pytest.raises(ValueError):
        qlinear.build_quant_linear(raw, TYPE_ID["Q4_K"], 4, 256)
    assert not qlinear.kernel_available(torch.device("cpu"))


def test_quantizable_table():
    assert qlinear.quantizable(TYPE_ID["Q4_0"], 4096, 4096)
    assert qlinear.quantizable(TYPE_ID["Q8_0"], 4096, 4096)
    assert not qlinear.quantizable(TYPE_ID["Q4_0"], 8, 32)                  # below min_elements
    assert qlinear.quantizable(TYPE_ID["Q4_0"], 8, 32, min_elements=0)
    assert not qlinear.quantizable(TYPE_ID["IQ2_XXS"], 4096, 4096)         # stays packed
    assert not qlinear.quantizable(3, 4096, 4096)                           # Q4_1: no kernel here
    with pytest.raises(ValueError):
        qlinear.build_quant_linear(torch.zeros(18, dtype=torch.uint8), 3, 1, 32)


def test_dispatch_constants():
    assert set(mmvq.FORMATE) == set(FORMATS)
    assert all(mmvq.MMVQ_BIS[f] == 16 and mmvq.MMQ_BIS[f] == 112 for f in FORMATS)
    assert cudakern.mm_bis("cpu") == 1 and cudakern.MM_ZEILEN == 16
    # every format stays in block format here (no int4 repack), so the reference's loader keeps expert
    # tensors of all of them as PackedExperts
    assert cudakern.IMMER_GEPACKT == frozenset(FORMATS)


def _route_reference(logits, k, normalize):
    """Restatement of the softmax branch of baukasten._auswahl (models/baukasten.py:171-190)."""
    p = torch.softmax(logits.float(), dim=-1)
    idx = p.topk(k, dim=-1)[1]
    w = p.gather(-1, idx)
    if normalize:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return idx, w


@pytest.mark.parametrize("normalize", [True, False])
def test_router(normalize):
    logits = synth.router_logits(16, 128, seed=4)
    idx, w = moe.route(logits, 8, normalize=normalize, weights_scale=2.0)
    ri, rw = _route_reference(logits, 8, normalize)
    assert torch.equal(idx, ri)
    assert torch.allclose(w, rw * 2.0)
    assert idx.shape == (16, 8) and idx.dtype == torch.int64


@pytest.mark.parametrize("fmt", list(FORMATS))
def test_synth_layout_and_size(fmt):
    bv, _ = FORMATS[fmt]
    n_in = 2 * 256
    raw = synth.blocks(fmt, 5, n_in, seed=9)
    assert raw.dtype == torch.uint8 and raw.numel() == 5 * row_bytes(fmt, n_in)
    assert torch.equal(raw, synth.blocks(fmt, 5, n_in, seed=9))          # seeded
    w = O.dequant(fmt, raw.numpy(), 5 * n_in)
    assert np.isfinite(w).all() and np.abs(w).max() > 0


def test_synth_q4k_scale_packing_round_trips():
    """pack_scale_min_k4 inverts the 6-bit unpacking of quant.py:99-108."""
    sc = torch.randint(0, 64, (50, 8))
    mn = torch.randint(0, 64, (50, 8))
    s = synth.pack_scale_min_k4(sc, mn).to(torch.int32)
    usc = torch.cat([s[:, 0:4] & 63, (s[:, 8:12] & 15) | ((s[:, 0:4] >> 6) << 4)], 1)
    umn = torch.cat([s[:, 4:8] & 63, (s[:, 8:12] >> 4) | ((s[:, 4:8] >> 6) << 4)], 1)
    assert torch.equal(usc, sc.to(torch.int32)) and torch.equal(umn, mn.to(torch.int32))


def test_synth_tq2_distribution():
    raw = synth.blocks("TQ2_0", 64, 4096, seed=1).view(-1, 66)[:, :64].to(torch.int32)
    codes = torch.stack([(raw >> (2 * g)) & 3 for g in range(4)]).flatten()
    freq = torch.bincount(codes, minlength=4).double() / codes.numel()
    assert abs(freq[0] - 0.3) < 0.01 and abs(freq[1] - 0.4) < 0.01 and abs(freq[2] - 0.3) < 0.01
    assert freq[3] == 0
