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


def test_exchange_kernels_match_the_tensor_path(cuda):
    """qmv_expert_dispatch / qmv_expert_combine give the layout and the sums of the tensor-operation path
    of ExpertShardedMoE (4 owners, ids out of range, bf16 input), bit for bit."""
    from nemicli_terminal_b200 import _lib, shard
    n_tok, k, n_exp, world, dim = 5, 3, 10, 4, 64
    g = torch.Generator().manual_seed(3)
    ids = torch.randint(0, n_exp, (n_tok, k), generator=g)
    ids[1, 2], ids[3, 0] = -1, n_exp + 3
    x = torch.randn(n_tok, dim, generator=g).to(torch.bfloat16)
    P = n_tok * k
    # the tensor path (shard.ExpertShardedMoE.dispatch on a CPU tensor)
    pe = ids.reshape(-1)
    valid = (pe >= 0) & (pe < n_exp)
    dest = torch.where(valid, shard.owner_of(pe.clamp(0, n_exp - 1), n_exp, world), torch.zeros_like(pe))
    onehot = (dest[:, None] == torch.arange(world)[None, :]).to(torch.int64)
    pos = (onehot.cumsum(0) - 1).gather(1, dest[:, None]).squeeze(1)
    slot_ref = dest * P + pos
    lo = torch.tensor([shard.shard_range(n_exp, world, r)[0] for r in range(world)])
    id_ref = torch.full((world * P,), -1.0)
    id_ref[slot_ref] = torch.where(valid, pe - lo[dest], torch.full_like(pe, -2)).float()
    lib = _lib.load()
    send = torch.full((world * P, dim + 4), 7.0, device=cuda)
    slot = torch.empty(P, dtype=torch.int64, device=cuda)
    sent = torch.empty(world, dtype=torch.int32, device=cuda)
    idc, xc = ids.reshape(-1).to(cuda), x.to(cuda)
    _lib.check(lib.qmv_expert_dispatch(_lib.ptr(idc), n_tok, k, n_exp, world, _lib.ptr(xc), 0, dim, _lib.ptr(send),
                                       dim + 4, _lib.ptr(slot), _lib.ptr(sent), _lib.stream_ptr(cuda)), "dispatch")
    send = send.cpu()
    assert torch.equal(slot.cpu(), slot_ref)
    assert torch.equal(send[:, dim], id_ref)
    assert torch.equal(sent.cpu().long(), onehot.sum(0))
    assert torch.equal(send[slot_ref, :dim], x.float()[torch.arange(P) // k])
    assert torch.count_nonzero(send[slot_ref, dim + 1:]) == 0
    y = torch.randn(world * P, dim, generator=g)
    w = torch.rand(n_tok, k, generator=g)
    out = torch.empty(n_tok, dim, device=cuda)
    yc, wc, sc = y.to(cuda), w.to(cuda), slot_ref.to(cuda)
    _lib.check(lib.qmv_expert_combine(_lib.ptr(yc), dim, _lib.ptr(sc), _lib.ptr(wc), n_tok, k, dim, _lib.ptr(out),
                                      _lib.stream_ptr(cuda)), "combine")
    assert torch.equal(out.cpu(), shard.combine(y[slot_ref].view(n_tok, k, dim), w))
