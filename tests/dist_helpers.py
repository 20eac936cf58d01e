"""Worker for the world-size-2 gloo tests of nemicli_terminal_b200.shard (CPU only).

The local products are injected (the CUDA kernels need a GPU): row shards use the oracle's
dequantise-and-multiply on real GGUF block bytes, expert shards a float64 expert FFN.  Each check
compares the sharded result on every rank with the unsharded computation of the same inputs."""
from __future__ import annotations

import os
import sys
import traceback

import torch
import torch.distributed as dist
import torch.nn.functional as F

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _expert_weights(n_exp, dim, ff, seed=3):
    g = torch.Generator().manual_seed(seed)
    wg = torch.randn(n_exp, ff, dim, generator=g, dtype=torch.float64) / dim ** 0.5
    wu = torch.randn(n_exp, ff, dim, generator=g, dtype=torch.float64) / dim ** 0.5
    wd = torch.randn(n_exp, dim, ff, generator=g, dtype=torch.float64) / ff ** 0.5
    return wg, wu, wd


def _ffn_ref(wg, wu, wd, ids, a):
    """Per pair: down_e(silu(gate_e a) * up_e a) in float64 -> float32."""
    out = []
    for e, v in zip(ids.tolist(), a.double()):
        if e < 0:                                                    # unused exchange slot
            out.append(torch.zeros(wd.shape[1], dtype=torch.float64))
            continue
        h = F.silu(wg[e] @ v) * (wu[e] @ v)
        out.append(wd[e] @ h)
    return torch.stack(out).float() if out else torch.zeros(0, wd.shape[1])


def check_rows(rank, world):
    from nemicli_terminal_b200 import shard, synth
    from oracle import oracle as O
    fmt, n_rows, n_in, M = "Q8_0", 301, 256, 3
    raw = synth.blocks(fmt, n_rows, n_in, seed=11)                   # same bytes on every rank
    x = synth.activations(M, n_in, seed=12)
    lo, hi = shard.shard_range(n_rows, world, rank)
    local = shard.slice_rows(fmt, raw, n_rows, n_in, lo, hi)

    def mv(raw_l, x2):
        return torch.from_numpy(O.mv_exact(fmt, raw_l.numpy(), hi - lo, n_in, x2.numpy())).float()

    lin = shard.RowShardedLinear(fmt, local, n_rows, n_in, matvec=mv)
    y = lin(x)
    ref = torch.from_numpy(O.mv_exact(fmt, raw.numpy(), n_rows, n_in, x.numpy())).float()
    assert y.shape == (M, n_rows), y.shape
    assert float((y - ref).abs().max()) <= 1e-6 * float(ref.abs().max()), "row shard differs"
    y1 = lin(x[0])                                                    # one token as a vector
    assert y1.shape == (n_rows,) and torch.equal(y1, y[0])


def check_bad_ids(rank, world):
    """Expert ids outside [0, n_exp) (-1, n_exp, a large one) add nothing to their token's sum."""
    from nemicli_terminal_b200 import shard, synth
    n_exp, dim, ff, L, k = 8, 64, 48, 4, 3
    wg, wu, wd = _expert_weights(n_exp, dim, ff)
    lo, hi = shard.shard_range(n_exp, world, rank)
    x = synth.activations(L, dim, seed=40 + rank)
    idx = torch.tensor([[0, -1, 7], [n_exp, 3, 5], [2, 6, 1000], [-1, n_exp, 4]])
    w = torch.rand(L, k, generator=torch.Generator().manual_seed(41 + rank))

    def ffn(local_ids, a):
        return _ffn_ref(wg, wu, wd, torch.where(local_ids >= 0, local_ids + lo, local_ids), a)

    y = shard.ExpertShardedMoE(None, None, None, n_exp, dim, ffn=ffn)(x, idx, w)
    ok = (idx >= 0) & (idx < n_exp)
    pairs = _ffn_ref(wg, wu, wd, torch.where(ok, idx, -1).reshape(-1), x.repeat_interleave(k, 0)).view(L, k, dim)
    assert torch.equal(y, shard.combine(pairs, w)), "refused expert ids changed the result"


def check_experts(rank, world, skew):
    from nemicli_terminal_b200 import moe, shard, synth
    n_exp, dim, ff, L, k = 8, 64, 48, 5, 2
    wg, wu, wd = _expert_weights(n_exp, dim, ff)
    lo, hi = shard.shard_range(n_exp, world, rank)
    x = synth.activations(L, dim, seed=20 + rank)                    # this rank's own tokens
    logits = synth.router_logits(L, n_exp, seed=30 + rank)
    if skew:                                                          # every pair to rank 0's experts
        logits[:, :shard.shard_range(n_exp, world, 0)[1]] += 100.0
    idx, w = moe.route(logits, k)

    def ffn(local_ids, a):
        return _ffn_ref(wg, wu, wd, torch.where(local_ids >= 0, local_ids + lo, local_ids), a)

    moe_layer = shard.ExpertShardedMoE(None, None, None, n_exp, dim, ffn=ffn)
    y = moe_layer(x, idx, w)
    pairs = _ffn_ref(wg, wu, wd, idx.reshape(-1), x.repeat_interleave(k, 0)).view(L, k, dim)
    ref = shard.combine(pairs, w)
    assert torch.equal(y, ref), f"expert shard differs by {float((y - ref).abs().max())}"
    if skew:                                     # pairs sent to each owner: all go to rank 0
        got = moe_layer.last_sent.tolist()
        assert got == [L * k] + [0] * (world - 1), got


def worker(rank, world, port, result_dir):
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    status = "ok"
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world)
        check_rows(rank, world)
        check_experts(rank, world, skew=False)
        check_experts(rank, world, skew=True)
        check_bad_ids(rank, world)
        dist.barrier()
    except Exception:                                                  # reported to the parent test
        status = traceback.format_exc()
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(status)


def gpu_worker(rank, world, port, result_dir):
    """Two NCCL ranks, one GPU each: vocab rows and experts sharded, every rank's result compared with
    the unsharded CUDA computation of the same inputs on that rank."""
    sys.path.insert(0, ROOT)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    status = "ok"
    try:
        import datetime
        from nemicli_terminal_b200 import mmvq, moe, shard, synth
        from nemicli_terminal_b200.formats import TYPE_ID
        from nemicli_terminal_b200.layers import PackedExperts
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        fmt, n_rows, n_in = "Q8_0", 16032 * world + 7, 4096
        raw = synth.blocks(fmt, n_rows, n_in, seed=50, device=dev)
        x = synth.activations(2, n_in, seed=51, device=dev)
        lo, hi = shard.shard_range(n_rows, world, rank)
        lin = shard.RowShardedLinear(fmt, shard.slice_rows(fmt, raw, n_rows, n_in, lo, hi), n_rows, n_in)
        y = lin(x)
        ref = mmvq.mv(fmt, raw, x, n_rows, n_in)
        assert torch.equal(y, ref), "row shard differs from the unsharded matvec"
        n_exp, dim, ff, L, k = 16, 2048, 768, 3, 8
        blobs = [synth.blocks("Q4_K", n_exp * o, i, seed=60 + s, device=dev) for s, (o, i) in
                 enumerate(((ff, dim), (ff, dim), (dim, ff)))]
        per = [b.numel() // n_exp for b in blobs]
        elo, ehi = shard.shard_range(n_exp, world, rank)
        mk = lambda b, p, o, i, a, e: PackedExperts(b[a * p:e * p].contiguous(), TYPE_ID["Q4_K"], e - a, o, i,  # noqa: E731
                                                     torch.float32)
        shapes = ((ff, dim), (ff, dim), (dim, ff))
        local = [mk(b, p, o, i, elo, ehi) for b, p, (o, i) in zip(blobs, per, shapes)]
        full = [mk(b, p, o, i, 0, n_exp) for b, p, (o, i) in zip(blobs, per, shapes)]
        xt = synth.activations(L, dim, seed=70 + rank, device=dev)
        idx, w = moe.route(synth.router_logits(L, n_exp, seed=80 + rank, device=dev), k)
        y = shard.ExpertShardedMoE(*local, n_exp, dim)(xt, idx, w)
        ref = moe.MoeFFN(*full)(xt, idx, w)
        assert float((y - ref).abs().max()) <= 1e-5 * float(ref.abs().max()), "expert shard differs"
        dist.barrier()
    except Exception:                                                  # reported to the parent test
        status = traceback.format_exc()
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()
    with open(os.path.join(result_dir, f"rank{rank}.txt"), "w") as f:
        f.write(status)
