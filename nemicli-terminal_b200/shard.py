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

Both exchanges have fixed sizes (the expert exchange sends fixed-capacity blocks with unused slots
marked), so nothing is read on the host and both calls can be captured in a CUDA graph.  Remote bytes
always arrive through the collective into this GPU's memory before a kernel reads them.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist
import torch.nn.functional as F

from . import _lib, mmvq, moe
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
        self._custom_mv = matvec is not None
        self._mv = matvec or self._mv_default

    def _mv_default(self, raw: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        return mmvq.mv(self.fmt, raw, x, self.n_local, self.n_in).reshape(-1, self.n_local)

    def local(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's outputs: (M, n_in) -> (M, n_local) float32."""
        x2 = x.reshape(-1, self.n_in)
        if self.n_local == 0:
            return torch.zeros(x2.shape[0], 0, dtype=torch.float32, device=x2.device)
        return self._mv(self.raw, x2).reshape(x2.shape[0], self.n_local)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        """(M, n_in) or (n_in,) -> (M, n_rows) or (n_rows,) float32 on every rank.

        The local product is written straight into this rank's block of the gather buffer
        [rank][token][n_pad] and gathered in place, so nothing is copied around the collective; with equal
        shards and one token the gathered buffer is the result itself."""
        x2 = x.reshape(-1, self.n_in)
        M = x2.shape[0]
        if self.world == 1:
            out = self.local(x2)
            return out.reshape(self.n_rows) if x.dim() == 1 else out
        buf = torch.empty(self.world, M, self.n_pad, dtype=torch.float32, device=x2.device)
        mine = buf[self.rank]
        if self.n_local == self.n_pad and not self._custom_mv:
            mmvq.mv(self.fmt, self.raw, x2 if M > 1 else x2[0], self.n_local, self.n_in, out=mine)
        elif self.n_local > 0:
            mine[:, :self.n_local] = self.local(x2)
        dist.all_gather_into_tensor(buf.view(-1), mine.reshape(-1), group=self.group)
        if self.n_rows == self.world * self.n_pad:                    # equal shards: no padding to drop
            out = buf.permute(1, 0, 2).reshape(M, self.n_rows) if M > 1 else buf.view(1, self.n_rows)
        else:
            sizes = [shard_range(self.n_rows, self.world, r) for r in range(self.world)]
            out = torch.cat([buf[r, :, :hi - lo] for r, (lo, hi) in enumerate(sizes)], 1)
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
    ffn(local_ids, a) -> (P, E) float32: optional replacement of the local expert computation.  The
    default with the SiLU gate and at most moe.GROUPED_UP_TO received rows is the grouped expert FFN
    (moe.grouped_ffn: every local expert read once per call, one slot per received row); otherwise
    gate/up -> act -> down run through the expert matvecs, each pair on its own input.  Ids of -1 mark unused
    slots, whose rows are ignored."""

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
        self._grouped = ffn is None and act is None
        self._ones = {}                         # (device, slots) -> unit weights of the grouped owner call
        self.last_sent: Optional[torch.Tensor] = None
        self._lo_tab = {}                       # device -> first expert of every rank

    def _ffn_cuda(self, ids: torch.Tensor, a: torch.Tensor) -> torch.Tensor:
        g = self.gate.matvec_je(ids, a)
        u = self.up.matvec_je(ids, a)
        return self.down.matvec_je(ids, (self.act(g) * u).contiguous())

    def _a2a(self, send: torch.Tensor) -> torch.Tensor:
        if self.world == 1:
            return send
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)      # equal splits: world blocks
        return recv

    # Every rank sends every rank a block of C = L * k pair slots (the most pairs one owner can receive
    # from it).  A slot is one row of dim + 4 floats: the pair's activation, then its expert id (local to
    # the owner; -1 for an unused slot, -2 for an id outside [0, n_exp)) as an exact float.  One all-to-all
    # carries the pairs to their owners, one brings the results back; all sizes are fixed and nothing is
    # read on the host, so a whole call can be captured in a CUDA graph.
    _ID = 4                                      # columns after the activation (the id, then padding)

    def dispatch(self, x: torch.Tensor, idx: torch.Tensor):
        """This rank's pairs to their owners -> (received slots (world * L * k, dim + 4) float32, slot of
        every local pair in the send buffer (L * k,) int64)."""
        L, k = idx.shape
        dev = x.device
        P = L * k
        pair_e = idx.reshape(-1).to(torch.int64)
        if _lib.on_gpu(x):                       # two kernels (qmv_expert_dispatch), same layout as below
            xin = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
            xin = xin.contiguous()
            ids = pair_e.to(dev).contiguous()
            send = torch.empty(self.world * P, self.dim + self._ID, dtype=torch.float32, device=dev)
            slot = torch.empty(P, dtype=torch.int64, device=dev)
            sent = torch.empty(self.world, dtype=torch.int32, device=dev)
            _lib.check(_lib.load().qmv_expert_dispatch(_lib.ptr(ids), L, k, self.n_exp, self.world, _lib.ptr(xin),
                                                       int(xin.dtype == torch.float32), self.dim, _lib.ptr(send),
                                                       self.dim + self._ID, _lib.ptr(slot), _lib.ptr(sent),
                                                       _lib.stream_ptr(dev)), "qmv_expert_dispatch")
            self.last_sent = sent
            return self._a2a(send), slot
        # an id outside [0, n_exp) goes to rank 0 as local id -2: the owner's kernels refuse it (zero rows and
        # the device status bit, as the single-GPU path does) and its weight adds nothing
        valid = (pair_e >= 0) & (pair_e < self.n_exp)
        dest = torch.where(valid, owner_of(pair_e.clamp(0, self.n_exp - 1), self.n_exp, self.world),
                           torch.zeros_like(pair_e))
        onehot = (dest[:, None] == torch.arange(self.world, device=dev)[None, :]).to(torch.int64)
        pos = (onehot.cumsum(0) - 1).gather(1, dest[:, None]).squeeze(1)   # rank among pairs to that owner
        slot = dest * P + pos
        lo_tab = self._lo_tab.get(dev)
        if lo_tab is None:                      # built on the first call (before any graph capture)
            lo_tab = torch.tensor([shard_range(self.n_exp, self.world, r)[0] for r in range(self.world)],
                                  dtype=torch.int64, device=dev)
            self._lo_tab[dev] = lo_tab
        send = torch.zeros(self.world * P, self.dim + self._ID, dtype=torch.float32, device=dev)
        send[:, self.dim] = -1.0
        rows = torch.cat([x.float()[torch.arange(P, device=dev) // k],
                          torch.where(valid, pair_e - lo_tab[dest], torch.full_like(pair_e, -2)).float()[:, None],
                          torch.zeros(P, self._ID - 1, dtype=torch.float32, device=dev)], 1)
        send[slot] = rows
        self.last_sent = onehot.sum(0)          # pairs this rank sent to each owner (no collective)
        return self._a2a(send), slot

    def compute(self, recv: torch.Tensor) -> torch.Tensor:
        """The owner's part: gate/up -> act -> down for every received slot -> (slots, dim) float32, zero rows
        for unused slots."""
        ids = recv[:, self.dim].to(torch.int64)
        a = recv[:, :self.dim]
        if self._grouped and a.shape[0] <= moe.GROUPED_UP_TO and moe.grouped_ok(self.gate, self.up, self.down, a,
                                                                               a.shape[0], 1):
            # one slot per received row, unit weight: the grouped kernels read each local expert once and
            # leave unused and refused slots at zero
            key = (a.device, a.shape[0])
            ones = self._ones.get(key)
            if ones is None:
                ones = self._ones[key] = torch.ones(a.shape[0], 1, dtype=torch.float32, device=a.device)
            return moe.grouped_ffn(self.gate, self.up, self.down, a, ids.view(-1, 1), ones)
        y = self._ffn(ids, a.contiguous()).float()
        return torch.where(ids[:, None] >= 0, y, torch.zeros_like(y))

    def __call__(self, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x (L, dim) this rank's tokens, idx (L, k) expert ids, w (L, k) weights -> (L, dim) float32: two
        all-to-alls (pairs out, results back) around the owners' expert FFNs, then the weighted sum in
        slot order on the home rank."""
        L, k = idx.shape
        recv, slot = self.dispatch(x, idx)
        y_back = self._a2a(self.compute(recv).contiguous())
        if _lib.on_gpu(y_back):                  # one kernel (qmv_expert_combine), the order of combine()
            wf = w.reshape(-1).to(device=y_back.device, dtype=torch.float32).contiguous()
            out = torch.empty(L, self.dim, dtype=torch.float32, device=y_back.device)
            _lib.check(_lib.load().qmv_expert_combine(_lib.ptr(y_back), self.dim, _lib.ptr(slot), _lib.ptr(wf), L, k,
                                                      self.dim, _lib.ptr(out), _lib.stream_ptr(y_back.device)),
                       "qmv_expert_combine")
            return out
        return combine(y_back[slot].view(L, k, self.dim), w)


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

