"""Multi-GPU sharding (nemicli_terminal_b200.shard): partition helpers in one process, and the
row-shard all-gather and expert-shard all-to-all exchanges as two gloo ranks on the CPU."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from nemicli_terminal_b200 import shard

import dist_helpers


def test_shard_range_covers_every_row_once():
    for n in (0, 1, 7, 128, 301, 128256):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    assert shard.shard_range(128256, 8, 3) == (48096, 64128)


def test_owner_matches_shard_range():
    for n_exp, world in ((128, 8), (8, 2), (10, 4), (3, 2)):
        e = torch.arange(n_exp)
        own = shard.owner_of(e, n_exp, world)
        for r in range(world):
            lo, hi = shard.shard_range(n_exp, world, r)
            assert (own[lo:hi] == r).all()


def test_expert_load_and_combine():
    idx = torch.tensor([[0, 5], [1, 7], [2, 3]])
    per, imb = shard.expert_load(idx, 8, 2)
    assert per == [4, 2] and abs(imb - 4 / 3) < 1e-12
    y = torch.arange(3 * 2 * 4, dtype=torch.float32).view(3, 2, 4)
    w = torch.tensor([[0.25, 0.75], [1.0, 0.0], [0.5, 0.5]])
    assert torch.allclose(shard.combine(y, w), (y * w.unsqueeze(-1)).sum(1))


def test_single_process_row_shard_is_the_whole_matrix():
    lin = shard.RowShardedLinear("Q8_0", torch.zeros(5 * 34, dtype=torch.uint8), 5, 32,
                                 matvec=lambda raw, x: torch.ones(x.shape[0], 5))
    assert lin.world == 1 and lin.n_local == 5
    assert torch.equal(lin(torch.zeros(2, 32)), torch.ones(2, 5))
    with pytest.raises(ValueError):
        shard.RowShardedLinear("Q8_0", torch.zeros(10, dtype=torch.uint8), 5, 32, matvec=lambda r, x: x)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_row_and_expert_shards(tmp_path):
    world = 2
    mp.start_processes(dist_helpers.worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    for r in range(world):
        status = (tmp_path / f"rank{r}.txt").read_text()
        assert status == "ok", f"rank {r}:\n{status}"
