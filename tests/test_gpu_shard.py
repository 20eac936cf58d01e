"""Sharded layers on the GPU: one rank (the CUDA matvec inside RowShardedLinear / ExpertShardedMoE
against the unsharded API) and, on boxes with two GPUs, two NCCL ranks."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from nemicli_terminal_b200 import mmvq, moe, shard, synth
from nemicli_terminal_b200.formats import TYPE_ID
from nemicli_terminal_b200.layers import PackedExperts

import dist_helpers

pytestmark = pytest.mark.gpu


def test_row_shard_one_rank_is_mmvq(cuda):
    fmt, n_rows, n_in = "Q8_0", 5000, 4096
    raw = synth.blocks(fmt, n_rows, n_in, seed=5, device=cuda)
    x = synth.activations(1, n_in, seed=6, device=cuda)[0]
    lin = shard.RowShardedLinear(fmt, raw, n_rows, n_in)
    assert torch.equal(lin(x), mmvq.mv(fmt, raw, x, n_rows, n_in))


def _experts(cuda, n_exp, dim, ff, seed):
    mk = lambda n_out, n_in, s: PackedExperts(synth.blocks("Q4_K", n_exp * n_out, n_in, seed=seed + s, device=cuda),  # noqa: E731
                                            TYPE_ID["Q4_K"], n_exp, n_out, n_in, torch.float32)
    return mk(ff, dim, 1), mk(ff, dim, 2), mk(dim, ff, 3)


def test_expert_shard_one_rank_matches_moe_ffn(cuda):
    n_exp, dim, ff, L, k = 16, 2048, 768, 4, 8
    gate, up, down = _experts(cuda, n_exp, dim, ff, 40)
    x = synth.activations(L, dim, seed=41, device=cuda)
    idx, w = moe.route(synth.router_logits(L, n_exp, seed=42, device=cuda), k)
    ref = moe.MoeFFN(gate, up, down)(x, idx, w)
    y = shard.ExpertShardedMoE(gate, up, down, n_exp, dim)(x, idx, w)
    assert float((y - ref).abs().max()) <= 1e-5 * float(ref.abs().max())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_nccl_ranks(tmp_path):
    world = 2
    mp.start_processes(dist_helpers.gpu_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        status = (tmp_path / f"rank{r}.txt").read_text()
        assert status == "ok", f"rank {r}:\n{status}"
