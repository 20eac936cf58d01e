"""The tensor-core tile path (qmv_mm_tc, tcgen05 kind::f16 with the accumulator in tensor memory) for
16..128+ tokens, against oracle C (the reference MMQ's fp16 arithmetic, ggufengine/mmvq.py:536-724,
summed exactly) and oracle A (dequantise + fp64 matmul).  Covers ragged row tiles, token counts that are
not a multiple of 16, more than one 128-token group, bf16 input, one K part and many, and run-to-run
equality (the split-K parts are added in a fixed order)."""
import numpy as np
import pytest
import torch

from nemicli_terminal_b200 import _lib, mmvq, synth
from nemicli_terminal_b200.formats import TYPE_ID
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case(fmt, n_out, n_in, M, cuda, seed=0, dtype=torch.float32):
    raw = synth.blocks(fmt, n_out, n_in, seed=seed + M, device=cuda)
    x = synth.activations(M, n_in, seed=seed + M + 1, device=cuda).to(dtype)
    return raw, x


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
@pytest.mark.parametrize("n_out,n_in", [(4096, 4096), (300, 2048), (1024, 14336)])
@pytest.mark.parametrize("M", [16, 17, 64, 112])
def test_tc_parity(cuda, fmt, n_out, n_in, M):
    raw, x = _case(fmt, n_out, n_in, M, cuda)
    y = mmvq.mm_tc(fmt, raw, x, n_out, n_in)
    assert y.shape == (M, n_out)
    yc = O.mmq(fmt, raw.cpu().numpy(), n_out, n_in, x.cpu().numpy())
    assert O.max_rel(y.cpu().numpy(), yc) < 2e-5
    ya = O.mv_exact(fmt, raw.cpu().numpy(), n_out, n_in, x.cpu().numpy())
    assert O.max_rel(y.cpu().numpy(), ya) < 1e-3
    assert torch.equal(y, mmvq.mm_tc(fmt, raw, x, n_out, n_in))


@pytest.mark.parametrize("fmt", ["Q4_K", "Q6_K"])
def test_tc_token_groups_and_bf16(cuda, fmt):
    """130 tokens: a group of 128 and one of 2; bf16 tokens read as the reference reads them."""
    n_out, n_in = 512, 4096
    raw, x = _case(fmt, n_out, n_in, 130, cuda, seed=7, dtype=torch.bfloat16)
    y = mmvq.mm_tc(fmt, raw, x, n_out, n_in)
    yc = O.mmq(fmt, raw.cpu().numpy(), n_out, n_in, x.float().cpu().numpy())
    assert O.max_rel(y.cpu().numpy(), yc) < 2e-5
    # each token's row depends on that token only (up to the fp32 order of another K partition)
    y1 = mmvq.mm_tc(fmt, raw, x[129:130], n_out, n_in)
    assert O.max_rel(y1.cpu().numpy(), y[129:130].cpu().numpy()) < 1e-5      # another K partition


def test_tc_single_part(cuda):
    """A matrix with enough row tiles to fill the SMs runs with one K part (no workspace sums)."""
    n_out, n_in = 65536, 1024
    raw, x = _case("Q4_K", n_out, n_in, 32, cuda, seed=11)
    y = mmvq.mm_tc("Q4_K", raw, x, n_out, n_in)
    yc = O.mmq("Q4_K", raw.cpu().numpy(), n_out, n_in, x.cpu().numpy())
    assert O.max_rel(y.cpu().numpy(), yc) < 2e-5


def test_tc_refusals(cuda):
    lib = _lib.load()
    assert lib.qmv_mm_tc_workspace_bytes(TYPE_ID["Q8_0"], 1024, 4096, 32) == 0
    assert lib.qmv_mm_tc_workspace_bytes(TYPE_ID["Q4_K"], 1024, 4000, 32) == 0
    raw, x = _case("Q8_0", 256, 256, 32, cuda)
    with pytest.raises(RuntimeError):
        mmvq.mm_tc("Q8_0", raw, x, 256, 256)
