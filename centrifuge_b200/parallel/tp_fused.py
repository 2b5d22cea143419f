"""Tensor-parallel collectives fused with their compute over NVLink / NVSwitch (sm_100a).

Sequence-parallel Megatron layers move activations with an all-gather before every
column-parallel GEMM and a reduce-scatter after every row-parallel GEMM (reference:
model/megatronlm.py:64-99, 152-178; those run as separate NCCL kernels).  Here both happen
inside the GEMM kernel (``gemm_tp``, csrc/kernels/gemm_sm100.cu), in one cooperative launch:

* all-gather (mode 1): the producer (RMSNorm forward or backward) writes the rank's rows into
  its own copy of a symmetric gather buffer; two extra warps per CTA of the consuming GEMM copy
  them to every other rank (one multicast store per 16 bytes through the NVSwitch, or peer
  stores) and raise a ready flag there, while the tensor cores start on the local rows (the m
  blocks are rotated so the own segment comes first); the TMA producer reads another rank's
  rows only after its flag;
* reduce-scatter (mode 2): the epilogue writes partial tiles into this rank's symmetric partial
  buffer and, when a 128-row block is complete, raises a per-block flag at the block's owners;
  two extra warps per CTA of every owner reduce its rows block by block as soon as all ranks
  have stored the block (``multimem.ld_reduce`` through the NVSwitch with fp32 accumulation, or
  peer loads), add the residual and write the layer output.  In the forward (uniform shards)
  the m-blocks are interleaved across owners so every owner pulls while the GEMM runs.

Rows are split into per-rank segments (:class:`Segments`): uniform sequence-parallel shards in
the forward, each rank's kept rows (compact global order) in the filtered backward, so the
GEMMs see exactly the kept rows.  Buffers live in ``torch.distributed._symmetric_memory``.  The
gather buffers are per call site ("slots", two per layer) and double as the saved activations
of the backward, so a slot is rewritten only by a later micro-batch's forward: the model keeps
one set of slots per micro-batch that can be in flight (one without pipelining, ``pp`` in a 1F1B
pipeline stage, whose TP group is then the stage's subgroup); the receive
partial buffers alternate by epoch and a GEMM of epoch e waits until every rank finished
reading epoch e - 2.  Flags carry monotonically increasing epochs (never reset); every rank issues the same
sequence of fused calls, so epochs agree across the group.  All waits are bounded (20 s) and
report through the kernels' error word.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from ..ops import fused
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
        self.nblk = (T + 127) // 128
        self.flags = symm_mem.empty(3 * P + self.nblk * P, dtype=torch.int32, device=self.device)
        self.flags.zero_()
        self.fhdl = symm_mem.rendezvous(self.flags, tp.group)
        self.peer_flags_dev = int(self.fhdl.buffer_ptrs_dev)
        # flag layout: gather ready[P] at 0, (unused) [P] at P, reduce-scatter done[P] at 2P,
        # reduce-scatter block ready[nblk][P] at 3P
        self.off_rs_done, self.off_blk = 2 * P, 3 * P
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
        self.cnt = torch.zeros(max(P, self.nblk) + 2, dtype=torch.int32, device=self.device)
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

    # ---------------------------------------------------------------- all-gather
    def rmsnorm_local(self, x_local: torch.Tensor, w: torch.Tensor, eps: float,
                      slot: int) -> Tuple[torch.Tensor, torch.Tensor]:
        """RMSNorm of this rank's shard written into its rows of gather slot ``slot``.

        Returns ``(slot [T, H] view, rstd [shard])``; the other ranks' rows arrive during the
        consuming :meth:`gemm_ag`."""
        seg = self.uniform_segments()
        xg = self.gather_view(slot)
        r0 = seg.start[self.rank]
        _, rstd = fused.rmsnorm_fwd(x_local, w, eps, out=xg[r0:r0 + self.shard])
        return xg, rstd

    def place_rows(self, rows_local: torch.Tensor, slot: int, seg: "Segments") -> torch.Tensor:
        """Write this rank's segment (first ``count`` local rows) into slot ``slot``; returns
        the slot view of the ``seg.total`` gathered rows."""
        xg = self.gather_view(slot, seg.total)
        r0, n = seg.start[self.rank], seg.counts[self.rank]
        if n:
            xg[r0:r0 + n].copy_(rows_local[:n])
        return xg

    def gemm_ag(self, xg: torch.Tensor, w: torch.Tensor, slot: int,
                rope: Optional[Tuple[torch.Tensor, torch.Tensor, int, int]] = None,
                seg: Optional["Segments"] = None, b_mn: bool = False,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """``xg @ w^T`` (``xg @ w`` with ``b_mn``) for a gather slot whose own rows are in place:
        the kernel all-gathers the other segments while it computes."""
        seg = seg or self.uniform_segments()
        N = w.shape[1] if b_mn else w.shape[0]
        if out is None:
            out = torch.empty(xg.shape[0], N, dtype=xg.dtype, device=self.device)
        self.ag_epoch += 1
        if xg.shape[0] == 0:
            return out
        pos, table, rc, hd = rope if rope is not None else (None, None, 0, 0)
        rot = (seg.start[self.rank] // 128) * 128
        T, H = self.T, self.H
        kernels().gemm_tp(xg, w, out, b_mn, pos, table, rc, hd, 1, self.rank, self.P, seg.dev,
                          self.ag_epoch, self.peer_flags_dev, 0, 0, self.cnt, rot,
                          self._mc(self.g_mc, slot * T * H), self.g_peers[slot].data_ptr(), 0, 0,
                          0, 0, None, None)
        return out

    # ---------------------------------------------------------------- reduce-scatter
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
        if T == 0:
            out.zero_()
            return out
        spb = (self.shard // 128) if seg is self._uniform and T == self.T else 0
        mc = self._mc(self.p_mc, i * self.T * self.H)
        kernels().gemm_tp(a, w, part, b_mn, None, None, 0, 0, 2, self.rank, self.P, seg.dev, e,
                          self.peer_flags_dev, 0, self.off_rs_done, self.cnt, 0, 0, 0, mc,
                          self.p_peers[i].data_ptr(), self.off_blk, spb, resid, out)
        return out


class VocabParallelCE:
    """Vocabulary-parallel cross entropy with the row statistics exchanged over NVLink.

    Replaces the three all-reduces (max, rescaled sum of exp, label logit) of the Megatron
    vocabulary-parallel loss (reference model/megatronlm.py:256-263): every rank writes its
    shard's per-row (max, sum exp, label logit) into its copy of a symmetric buffer (two slots,
    alternating by call), raises a ready flag at every rank, and one kernel per rank combines
    the P triples of each row into lse and loss after a bounded wait
    (``cfb_ce_exchange``).  A slot is rewritten two calls later, once every rank has reported
    (done flag) that it read it.  Every rank of the group makes the same sequence of calls."""

    def __init__(self, tp, T: int, device):
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        from ..ops._ext import status_block
        self.tp, self.P, self.rank, self.T = tp, tp.size, tp.rank, T
        self.device = torch.device(device)
        self.stats = symm_mem.empty(2 * 3 * T, dtype=torch.float32, device=self.device)
        self.shdl = symm_mem.rendezvous(self.stats, tp.group)
        self.flags = symm_mem.empty(2 * self.P, dtype=torch.int32, device=self.device)
        self.flags.zero_()
        self.fhdl = symm_mem.rendezvous(self.flags, tp.group)
        self.peer_flags_dev = int(self.fhdl.buffer_ptrs_dev)
        sb = [int(x) for x in self.shdl.buffer_ptrs]
        self.peers = [torch.tensor([b + i * 3 * T * 4 for b in sb], dtype=torch.int64,
                                   device=self.device) for i in range(2)]
        self.counter = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.err = status_block(self.device)
        self.epoch = 0
        torch.cuda.synchronize(self.device)
        dist.barrier(tp.group)

    def __call__(self, logits: torch.Tensor, labels: torch.Tensor, vocab_start: int):
        """``logits`` [T, V/P] bf16 of this rank's shard, ``labels`` [T] (global ids, < 0
        ignored); returns (loss [T], lse [T]) fp32, the same on every rank."""
        T, P = labels.numel(), self.P
        assert T <= self.T and labels.dtype == torch.long
        k = kernels()
        self.epoch += 1
        e, i = self.epoch, self.epoch & 1
        if e > 2:  # every rank has read this slot's previous contents
            k.symm_wait(self.flags.data_ptr(), P, 1, P, e - 2, self.err)
        st = self.stats[i * 3 * self.T:i * 3 * self.T + 3 * T].view(3, T)
        fused.ce_partial(logits, labels, vocab_start, out=(st[0], st[1], st[2]))
        # the exchange kernel indexes a slot as [3][T] of this call's T: offsets use T
        k.symm_signal(self.peer_flags_dev, P, self.rank, e)
        loss = torch.empty(T, dtype=torch.float32, device=self.device)
        lse = torch.empty_like(loss)
        k.ce_exchange(self.peers[i].data_ptr(), P, labels, loss, lse, self.flags.data_ptr(), 0,
                      e, self.peer_flags_dev, P, self.rank, self.counter, self.err)
        return loss, lse


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
