"""Tensor + sequence parallelism: process-group helpers and the kept-row layout.

Megatron-style TP (reference: model/megatronlm.py:46-279, ColumnParallelLinear /
RowParallelLinear) with sequence parallelism: the residual stream is sharded by token rows
(rank ``p`` of ``P`` owns rows ``[p*T/P, (p+1)*T/P)`` of the flattened ``[B*S, H]`` stream);
column-parallel GEMMs consume an all-gather of their normalised input, row-parallel GEMMs
produce partial sums that are reduce-scattered back to the row shards.

In the filtered backward only kept rows move between ranks.  A rank's shard keeps a
data-dependent number of rows, so the backward uses a padded layout: every rank holds ``C`` rows
(``C`` = the largest per-rank kept count, one host read per micro-batch), its real kept rows
first, zero rows after.  All-gathers and reduce-scatters then have equal sizes on every rank;
index maps convert between the padded layout ``[P*C]`` and the compact global kept order
``[Tk]`` (kept rows sorted by position, which is rank-major because shards are row ranges).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


class TPGroup:
    """Collectives of one tensor-parallel group (NCCL on GPU, gloo on CPU ranks)."""

    def __init__(self, group=None):
        self.group = group
        if dist.is_available() and dist.is_initialized():
            self.size = dist.get_world_size(group)
            self.rank = dist.get_rank(group)
        else:
            self.size, self.rank = 1, 0

    def all_gather_rows(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        out = torch.empty((self.size * x.shape[0],) + tuple(x.shape[1:]), dtype=x.dtype,
                          device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=self.group)
        return out

    def reduce_scatter_rows(self, x: torch.Tensor) -> torch.Tensor:
        if self.size == 1:
            return x
        out = torch.empty((x.shape[0] // self.size,) + tuple(x.shape[1:]), dtype=x.dtype,
                          device=x.device)
        dist.reduce_scatter_tensor(out, x.contiguous(), group=self.group)
        return out

    def all_reduce_(self, x: torch.Tensor, op=None) -> torch.Tensor:
        if self.size > 1:
            dist.all_reduce(x, op=op or dist.ReduceOp.SUM, group=self.group)
        return x


class KeptLayout:
    """Kept rows of a row-sharded ``[T, *]`` tensor, padded per rank to a common count.

    Attributes (int32 on the device):
      ``rows``      [Tk]    global kept rows (compact order)
      ``local``     [C]     this rank's kept rows as shard-local indices, padded with 0
      ``c2p``       [Tk]    compact index -> padded slot (owner * C + j)
      ``p2c``       [P*C]   padded slot -> compact index, or Tk for padding (a zero row)
      ``C``, ``count`` (this rank's real kept rows), ``Tk``, ``counts`` (host list, per rank)
    """

    def __init__(self, rows: Optional[torch.Tensor], T: int, tp: TPGroup, device):
        P, p = tp.size, tp.rank
        assert T % P == 0, f"{T} token rows are not divisible by TP={P}"
        shard = T // P
        i32 = dict(dtype=torch.int32, device=device)
        if rows is None:  # unfiltered: every row kept, no padding
            self.rows = torch.arange(T, **i32)
            self.Tk, self.C, self.count = T, shard, shard
            self.local = torch.arange(shard, **i32)
            self.c2p = self.rows
            self.p2c = self.rows
            self.counts = [shard] * P
            self.identity = True
            return
        self.identity = False
        rows = rows.to(device=device, dtype=torch.int64)
        Tk = rows.numel()
        if P == 1:  # one shard: the padded layout is the compact one, no host read
            self.rows = rows.to(torch.int32)
            self.Tk, self.C, self.count, self.counts = Tk, Tk, Tk, [Tk]
            self.local = self.rows
            self.c2p = torch.arange(Tk, **i32)
            self.p2c = self.c2p
            return
        owner = rows // shard
        counts = torch.bincount(owner, minlength=P)
        prefix = torch.cumsum(counts, 0) - counts
        cvals = counts.tolist()  # one host read per micro-batch
        C = max(cvals)
        j = torch.arange(Tk, device=device) - prefix[owner]
        c2p = owner * C + j
        p2c = torch.full((P * C,), Tk, dtype=torch.int64, device=device)
        p2c[c2p] = torch.arange(Tk, device=device)
        local = torch.zeros(C, dtype=torch.int64, device=device)
        mine = rows[owner == p] - p * shard
        local[:mine.numel()] = mine
        self.rows = rows.to(torch.int32)
        self.counts = cvals
        self.Tk, self.C, self.count = Tk, C, cvals[p]
        self.local = local.to(torch.int32)
        self.c2p = c2p.to(torch.int32)
        self.p2c = p2c.to(torch.int32)

    def to_compact(self, padded: torch.Tensor, gather) -> torch.Tensor:
        """``[P*C, H]`` (all-gathered padded rows) -> ``[Tk, H]``."""
        if self.identity:
            return padded
        return gather(padded, self.c2p)

    def to_padded(self, compact_plus_zero: torch.Tensor, gather) -> torch.Tensor:
        """``[Tk+1, H]`` (compact rows followed by one zero row) -> ``[P*C, H]``."""
        if self.identity:
            return compact_plus_zero[:self.Tk]
        return gather(compact_plus_zero, self.p2c)
