"""Multi-GPU sharding of the matvec path: row-sharded projections and expert-sharded MoE layers.

One process per GPU; torch.distributed carries the exchanges (NCCL between B200s over NVLink /
NVSwitch, gloo for the host-side tests).  The reference runs on one GPU only; its weights and call
signatures are kept (ggufengine/models/common.py:364-492, models/moe.py:264-321), the split is new:

RowShardedLinear   rank g holds rows [g*N/G, (g+1)*N/G) of an (N, n_in) block-format matrix (whole
                   GGUF rows, no block is split).  Every rank quantises the replicated input itself
                   and multiplies its slice; one all-gather of the fp32 outputs gives every rank all N
                   outputs.  For the vocabulary projection (128256 x 4096) at G = 8 that is 16032 rows
                   per GPU and 513 KB gathered per token.
ExpertShardedMoE   rank g holds experts [g*E/G, (g+1)*E/G).  Tokens stay on their home rank; each
                   (token, slot) pair's activation goes to the rank that owns the slot's expert
                   (all-to-all), the owner runs gate/up -> act -> down for the pairs it received,
                   the results come back (all-to-all) and the home rank forms the weighted sum in slot
                   order.

The exchanges take their sizes from the routing on the host (one device-to-host copy of the pair
counts per call), so an expert-sharded call is not captured in a CUDA graph; the row-sharded call is
(its sizes are fixed).  Remote bytes always arrive through the collective into this GPU's memory
before a kernel reads them.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import mmvq
from .formats import row_bytes
from .layers import PackedExperts


def _world(group) -> Tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def shard_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows (or experts) [lo, hi) of rank `rank` when n are split over `world` ranks as evenly as
    whole items allow (the first n % world ranks hold one more)."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def slice_rows(fmt: str, raw: torch.Tensor, n_rows: int, n_in: int, lo: int, hi: int) -> torch.Tensor:
    """Rows [lo, hi) of a flat block-format matrix (n_rows, n_in), as a contiguous flat tensor."""
    rb = row_bytes(fmt, n_in)
    flat = raw.reshape(-1)
    if flat.numel() != n_rows * rb:
        raise ValueError(f"slice_rows: {flat.numel()} bytes is not {n_rows} rows of {rb}")
    return flat[lo * rb:hi * rb].contiguous()


class RowShardedLinear:
    """y = x @ W^T for W (n_rows, n_in) in a block format, rows split over the ranks of `group`.

    raw_local: this rank's rows (shard_range(n_rows, world, rank)) as block bytes.  matvec(raw_local,
    x) -> (M, n_local) float32 is the local product; the default is this package's CUDA kernel
    (mmvq.mv), which refuses tensors that are not on a GPU."""

    def __init__(self, fmt: str, raw_local: torch.Tensor, n_rows: int, n_in: int, group=None,
                 matvec: Optional[Callable[[torch.Tensor, torch.Tensor], torch.Tensor]] = None):
        self.world, self.rank = _world(group)
        self.group = group
        self.fmt, self.n_rows, self.n_in = fmt, n_rows, n_in
        self.lo, self.hi = shard_range(n_rows, self.world, self.rank)
        self.n_local = self.hi - self.lo
        self.n_pad = -(-n_rows // self.world)                     # rows per rank in the gather buffer
        if raw_local.numel() != self.n_local * row_bytes(fmt, n_in):
            raise ValueError(f"RowShardedLinear: rank {self.rank} needs rows [{self.lo}, {self.hi}) "
                             f"({self.n_local * row_bytes(fmt, n_in)} bytes), got {raw_local.numel()}")
        self.raw = raw_local.reshape(-1)
        self._mv = matvec or (lambda raw, x: mmvq.mv(self.fmt, raw, x, self.n_local, self.n_in).reshape(-1, self.n_local))

    def local(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's outputs: (M, n_in) -> (M, n_local) float32."""
        x2 = x.reshape(-1, self.n_in)
        if self.n_local == 0:
            return torch.zeros(x2.shape[0], 0, dtype=torch.float32, device=x2.device)
        return self._mv(self.raw, x2).reshape(x2.shape[0], self.n_local)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """(M, n_in) or (n_in,) -> (M, n_rows) or (n_rows,) float32 on every rank."""
        x2 = x.reshape(-1, self.n_in)
        M = x2.shape[0]
        y = self.local(x2)
        if self.world == 1:
            out = y
        else:
            send = torch.zeros(self.n_pad, M, dtype=torch.float32, device=y.device)
            send[:self.n_local] = y.t()
            recv = torch.empty(self.world * self.n_pad, M, dtype=torch.float32, device=y.device)
            dist.all_gather_into_tensor(recv, send, group=self.group)
            parts = []
            for r in range(self.world):
                lo, hi = shard_range(self.n_rows, self.world, r)
                parts.append(recv[r * self.n_pad:r * self.n_pad + hi - lo])
            out = torch.cat(parts, 0).t().contiguous()
        return out.reshape(self.n_rows) if x.dim() == 1 else out


def owner_of(expert: torch.Tensor, n_exp: int, world: int) -> torch.Tensor:
    """Rank that holds each expert id under shard_range(n_exp, world, .)."""
    base, extra = divmod(n_exp, world)
    big = extra * (base + 1)                                        # experts held by the larger ranks
    e = expert.to(torch.int64)
    return torch.where(e < big, e // (base + 1), extra + (e - big) // max(base, 1))


class ExpertShardedMoE:
    """MoE FFN with the experts split over the ranks of `group`; tokens stay on their home rank.

    gate, up, down: this rank's experts (PackedExperts holding shard_range(n_exp, world, rank)).
    ffn(local_ids, a) -> (P, E) float32: optional replacement of the local expert computation (the
    default runs gate/up -> act -> down through the CUDA kernels, each pair on its own input)."""

    def __init__(self, gate: Optional[PackedExperts], up: Optional[PackedExperts], down: Optional[PackedExperts],
                 n_exp: int, dim: int, group=None, act: Optional[Callable] = None,
                 ffn: Optional[Callable[[torch.Tensor, torch.Tensor], torch.Tensor]] = None):
        self.world, self.rank = _world(group)
        self.group = group
        self.n_exp, self.dim = n_exp, dim
        self.lo, self.hi = shard_range(n_exp, self.world, self.rank)
        self.act = act or F.silu
        if ffn is None:
            for ex in (gate, up, down):
                if ex is None or ex.n_exp != self.hi - self.lo:
                    raise ValueError(f"ExpertShardedMoE: rank {self.rank} must hold experts [{self.lo}, {self.hi})")
            if gate.n_in != dim or down.n_out != dim or gate.n_out != up.n_out or down.n_in != gate.n_out:
                raise ValueError("ExpertShardedMoE: gate/up/down shapes do not chain")
        self.gate, self.up, self.down = gate, up, down
        self._ffn = ffn or self._ffn_cuda
        self.last_load: Optional[List[int]] = None

    def _ffn_cuda(self, ids: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
        g = self.gate.matvec_je(ids, a)
        u = self.up.matvec_je(ids, a)
        return self.down.matvec_je(ids, (self.act(g) * u).contiguous())

    def _exchange(self, send: torch.Tensor, send_counts: List[int], recv_counts: List[int]) -> torch.Tensor:
        recv = torch.empty((sum(recv_counts),) + tuple(send.shape[1:]), dtype=send.dtype, device=send.device)
        dist.all_to_all_single(recv, send, output_split_sizes=recv_counts, input_split_sizes=send_counts,
                               group=self.group)
        return recv

    def __call__(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x (L, dim) this rank's tokens, idx (L, k) expert ids, w (L, k) weights -> (L, dim) float32."""
        L, k = idx.shape
        dev = x.device
        pair_e = idx.reshape(-1).to(torch.int64)
        dest = owner_of(pair_e, self.n_exp, self.world)
        order = torch.argsort(dest * (L * k) + torch.arange(L * k, device=dev))   # by owner, stable
        send_counts_t = torch.bincount(dest, minlength=self.world)
        if self.world > 1:
            recv_counts_t = torch.empty_like(send_counts_t)
            dist.all_to_all_single(recv_counts_t, send_counts_t, group=self.group)
        else:
            recv_counts_t = send_counts_t
        send_counts = [int(c) for c in send_counts_t.cpu()]
        recv_counts = [int(c) for c in recv_counts_t.cpu()]
        self.last_load = recv_counts
        token = order // k
        a_send = x.float()[token].contiguous()                      # (L*k, dim), grouped by owner
        e_send = pair_e[order]
        if self.world > 1:
            a_recv = self._exchange(a_send, send_counts, recv_counts)
            e_recv = self._exchange(e_send, send_counts, recv_counts)
        else:
            a_recv, e_recv = a_send, e_send
        if e_recv.numel():
            y_recv = self._ffn((e_recv - self.lo).contiguous(), a_recv).float()
        else:
            y_recv = torch.zeros(0, self.dim, dtype=torch.float32, device=dev)
        y_back = self._exchange(y_recv.contiguous(), recv_counts, send_counts) if self.world > 1 else y_recv
        y_pairs = torch.empty(L * k, self.dim, dtype=torch.float32, device=dev)
        y_pairs[order] = y_back
        return combine(y_pairs.view(L, k, self.dim), w)


def combine(y: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """sum_j w[t, j] * y[t, j] accumulated in slot order: (L, k, dim), (L, k) -> (L, dim) float32."""
    out = y[:, 0] * w[:, 0:1].float()
    for j in range(1, y.shape[1]):
        out = out + y[:, j] * w[:, j:j + 1].float()
    return out


def expert_load(idx: torch.Tensor, n_exp: int, world: int) -> Tuple[List[int], float]:
    """(pairs per rank, max/mean) of a routing: the load imbalance an expert-sharded call sees."""
    per = torch.bincount(owner_of(idx.reshape(-1), n_exp, world), minlength=world).tolist()
    mean = sum(per) / world
    return per, (max(per) / mean if mean else 1.0)

