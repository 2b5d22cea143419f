"""Tensor-parallel collectives fused with their compute over NVLink / NVSwitch (sm_100a).

Sequence-parallel Megatron layers move activations with an all-gather before every
column-parallel GEMM and a reduce-scatter after every row-parallel GEMM (reference:
model/megatronlm.py:64-99, 152-178; those run as separate NCCL kernels).  Here both are fused
into the kernels that produce or consume the data:

* all-gather: the RMSNorm kernel of the rank's rows writes its output once into every rank's
  gather buffer through the NVSwitch multicast address (or peer stores without multicast) and
  raises per-shard ready flags; the column-parallel GEMM waits on each shard's flag inside its
  TMA producer and starts with its own shard (``gemm_tp`` mode 1, optionally with the RoPE
  epilogue), so the transfer of remote shards overlaps its math;
* reduce-scatter: the row-parallel GEMM writes partial sums into this rank's symmetric partial
  buffer and tells each shard's owner when that shard's tiles are stored; two extra warps per CTA
  of the same cooperative launch wait for the rank's own shard and pull it summed over all ranks
  (``multimem.ld_reduce`` with fp32 accumulation through the switch, or peer loads), add the
  residual and write the layer output (``gemm_tp`` mode 2).

Buffers live in ``torch.distributed._symmetric_memory`` (same offsets on every rank).  The
gather buffers are per call site ("slots", e.g. two per layer) and double as the saved
activations of the backward, so a slot is rewritten only by the next micro-batch's forward.  The
two partial buffers alternate by epoch; a GEMM of epoch e waits until every rank finished
pulling from epoch e - 2.  Flags carry monotonically increasing epochs (never reset); every rank
issues the same sequence of fused calls, so epochs agree across the group.  All waits are
bounded (20 s) and report through the kernels' error word.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ..ops._ext import kernels


class TPFusedComm:
    def __init__(self, tp, T: int, H: int, n_gather: int, device, use_multicast: bool = True):
        import torch.distributed._symmetric_memory as symm_mem
        self.tp = tp
        self.P, self.rank = tp.size, tp.rank
        assert T % self.P == 0 and (T // self.P) % 128 == 0, \
            f"{T} rows do not split into {self.P} shards of 128-row blocks"
        self.T, self.H, self.shard = T, H, T // self.P
        self.device = torch.device(device)
        bf16 = torch.bfloat16
        self.n_gather = n_gather
        self.gbuf = symm_mem.empty(n_gather * T * H, dtype=bf16, device=self.device)
        self.ghdl = symm_mem.rendezvous(self.gbuf, tp.group)
        self.pbuf = symm_mem.empty(2 * T * H, dtype=bf16, device=self.device)
        self.phdl = symm_mem.rendezvous(self.pbuf, tp.group)
        P = self.P
        self.flags = symm_mem.empty(3 * P, dtype=torch.int32, device=self.device)
        self.flags.zero_()
        self.fhdl = symm_mem.rendezvous(self.flags, tp.group)
        self.peer_flags_dev = int(self.fhdl.buffer_ptrs_dev)
        self.ag_ready = self.flags.data_ptr()  # local ready[P] of the gathers (offset 0)
        self.off_rs_ready, self.off_rs_done = P, 2 * P
        mc_ok = use_multicast and self.ghdl.has_multicast_support and self.phdl.has_multicast_support
        self.g_mc = int(self.ghdl.multicast_ptr) if mc_ok else 0
        self.p_mc = int(self.phdl.multicast_ptr) if mc_ok else 0
        gb = [int(x) for x in self.ghdl.buffer_ptrs]
        pb = [int(x) for x in self.phdl.buffer_ptrs]
        esz = 2
        # device arrays of the P peer addresses of every gather slot and partial buffer
        self.g_peers = [torch.tensor([b + s * T * H * esz for b in gb], dtype=torch.int64,
                                     device=self.device) for s in range(n_gather)]
        self.p_peers = [torch.tensor([b + i * T * H * esz for b in pb], dtype=torch.int64,
                                     device=self.device) for i in range(2)]
        self.cnt = torch.zeros(P + 2, dtype=torch.int32, device=self.device)
        self.push_cnt = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ag_epoch = 0
        self.rs_epoch = 0
        self._uniform = None
        torch.cuda.synchronize(self.device)
        import torch.distributed as dist
        dist.barrier(tp.group)

    @property
    def kind(self) -> str:
        return "nvls-multimem" if self.g_mc else "p2p"

    def gather_view(self, slot: int, rows: Optional[int] = None) -> torch.Tensor:
        T, H = self.T, self.H
        return self.gbuf[slot * T * H:(slot + 1) * T * H].view(T, H)[: (T if rows is None else rows)]

    def uniform_segments(self) -> "Segments":
        if self._uniform is None:
            counts = [self.shard] * self.P
            self._uniform = Segments(counts, self.device)
        return self._uniform

    def _mc(self, base: int, slot_elems: int) -> int:
        return base + slot_elems * 2 if base else 0

    # ---------------------------------------------------------------- all-gather producers
    def rmsnorm_push(self, x_local: torch.Tensor, w: torch.Tensor, eps: float,
                     slot: int) -> Tuple[torch.Tensor, torch.Tensor, int]:
        """RMSNorm of the local shard (uniform segments), gathered into slot ``slot``.

        Returns ``(gathered [T, H] view, rstd [shard], epoch)``; the gathered rows are complete
        only for a consumer that waits on ``epoch`` (:meth:`gemm_ag`)."""
        assert x_local.shape[0] == self.shard and x_local.shape[1] == self.H
        self.ag_epoch += 1
        rstd = torch.empty(self.shard, dtype=torch.float32, device=self.device)
        T, H = self.T, self.H
        kernels().tp_rmsnorm_push(x_local, w, eps, self._mc(self.g_mc, slot * T * H),
                                  self.g_peers[slot].data_ptr(), H, rstd, self.peer_flags_dev, 0,
                                  self.rank, self.P, self.rank * self.shard, self.ag_epoch,
                                  self.push_cnt)
        return self.gather_view(slot), rstd, self.ag_epoch

    def rmsnorm_bwd_push(self, dy, x, rstd, w, dw_acc, x_rows, dres, slot: int,
                         seg: "Segments") -> Tuple[torch.Tensor, torch.Tensor, int]:
        """RMSNorm backward of the local (padded) rows whose first ``count`` output rows are also
        gathered into slot ``slot`` at this rank's segment.  Returns ``(dx [rows, H],
        gathered [Tk, H] view, epoch)``."""
        self.ag_epoch += 1
        T, H = self.T, self.H
        dx = torch.empty_like(dy)
        partial_rows = max(1, min(dy.shape[0], 148 * 2))
        kernels().tp_rmsnorm_bwd_push(dy, x, x_rows, rstd, w, dres, dx, dw_acc, partial_rows,
                                      self._mc(self.g_mc, slot * T * H),
                                      self.g_peers[slot].data_ptr(), H, seg.start[self.rank],
                                      seg.counts[self.rank], self.peer_flags_dev, 0, self.rank,
                                      self.P, self.ag_epoch, self.push_cnt)
        return dx, self.gather_view(slot, seg.total), self.ag_epoch

    # ---------------------------------------------------------------- consumers / producers
    def gemm_ag(self, xg: torch.Tensor, w: torch.Tensor, epoch: int,
                rope: Optional[Tuple[torch.Tensor, torch.Tensor, int, int]] = None,
                seg: Optional["Segments"] = None, b_mn: bool = False,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``xg @ w^T`` (``xg @ w`` with ``b_mn``) where ``xg`` is a gathered slot, waiting per
        source segment inside the kernel."""
        seg = seg or self.uniform_segments()
        N = w.shape[1] if b_mn else w.shape[0]
        if out is None:
            out = torch.empty(xg.shape[0], N, dtype=xg.dtype, device=self.device)
        if xg.shape[0] == 0:
            return out
        pos, table, rc, hd = rope if rope is not None else (None, None, 0, 0)
        rot = (seg.start[self.rank] // 128) * 128
        kernels().gemm_tp(xg, w, out, b_mn, pos, table, rc, hd, 1, self.rank, self.P, seg.dev,
                          epoch, self.ag_ready, rot, 0, 0, 0, None, 0, 0, None, None)
        return out

    def gemm_rs(self, a: torch.Tensor, w: torch.Tensor, resid: Optional[torch.Tensor],
                seg: Optional["Segments"] = None, b_mn: bool = False,
                out_rows: Optional[int] = None, out: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
        """This rank's segment of ``sum_ranks(a @ w^T)`` (``a @ w`` with ``b_mn``) plus
        ``resid``, as ``[out_rows, N]`` (rows past the segment are zero)."""
        seg = seg or self.uniform_segments()
        T = a.shape[0]
        N = w.shape[1] if b_mn else w.shape[0]
        assert T == seg.total and T <= self.T and N <= self.H
        self.rs_epoch += 1
        e = self.rs_epoch
        i = e & 1
        part = self.pbuf[i * self.T * self.H:i * self.T * self.H + max(T, 1) * N].view(-1, N)[:T]
        rows = seg.counts[self.rank] if out_rows is None else out_rows
        if out is None:
            out = torch.empty(rows, N, dtype=a.dtype, device=self.device)
        kernels().gemm_tp(a, w, part, b_mn, None, None, 0, 0, 2, self.rank, self.P, seg.dev, e, 0,
                          0, self.peer_flags_dev, self.off_rs_ready, self.off_rs_done, self.cnt,
                          self._mc(self.p_mc, i * self.T * self.H), self.p_peers[i].data_ptr(),
                          resid, out)
        return out


class Segments:
    """Per-rank row segments of a sequence-parallel tensor: rank q owns rows
    ``[start[q], start[q] + counts[q])`` (host lists) and ``dev`` is the int32 device prefix
    array ``[P + 1]`` the kernels read."""

    def __init__(self, counts, device):
        self.counts = [int(c) for c in counts]
        self.start = [0]
        for c in self.counts:
            self.start.append(self.start[-1] + c)
        self.total = self.start[-1]
        self.dev = torch.tensor(self.start, dtype=torch.int32, device=device)
