"""Fused gradient reduce-scatter over NVLink peer memory (the ZeRO-2 product path).

The flat fp32 gradient buffer of every rank is allocated in symmetric memory
(``torch.distributed._symmetric_memory``: same offsets on every GPU, peer pointers, and an
NVSwitch multicast mapping when NVLS is available).  For each bucket the rank's own sm_100a
kernel (csrc/kernels/comm_sm100.cu) pulls its chunk from all ranks -- one
``multimem.ld_reduce.add.v4.f32`` per 16 bytes through the switch, or plain peer loads -- and
adds the sum into the rank's fp32 ZeRO-2 shard.  No cast pass, no staging buffer, no NCCL
kernel on this path; gradients travel as fp32 so the accumulation is exact.

Ordering uses per-bucket "ready" flags and a per-micro-batch "done" flag in a small
symmetric flag buffer, written with release stores and waited on with bounded acquire spins
(timeout -> the device status block's error word, never a trap).  The local gradient buffer is
cleared only after every rank has finished reading it; after a failed wait the pull and the
clear are skipped on the device and the step's AdamW update too (the trainer's
:class:`~centrifuge_b200.utils.device_status.DeviceStatus` raises one step later).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import kernels, status_block

MAX_BUCKETS = 4096


class SymmReducer:
    """``ring=True``: partitioned ZeRO-2 (the optimizer's gradient ring lives in symmetric
    memory, allocated through :meth:`alloc_ring`; after pulling a bucket each rank raises a
    per-bucket "pulled" flag at every peer, and a slot is written again only once every peer
    has pulled it).  Otherwise the model's full fp32 gradient buffer moves to symmetric memory."""

    def __init__(self, flat, group, use_multicast: bool = True, ring: bool = False):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group
        self.W = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.ring = ring
        self.use_multicast = use_multicast
        dev = flat.device
        self.device = dev
        self.flat = flat
        nflags = 2 * MAX_BUCKETS * self.W + 2 * self.W  # ready, done + param, pulled
        self.flags = symm_mem.empty(nflags, dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.fhdl = symm_mem.rendezvous(self.flags, group)
        self.peer_flags_dev = int(self.fhdl.buffer_ptrs_dev)
        nvls = use_multicast and self.fhdl.has_multicast_support
        self.mc = 0
        self.peer_ptrs_dev = 0
        self.base_ptr = 0
        if not ring:
            buf = symm_mem.empty(flat.numel, dtype=torch.float32, device=dev)
            flat.rebind_grad(buf)
            self.hdl = symm_mem.rendezvous(buf, group)
            self.mc = int(self.hdl.multicast_ptr) if (nvls and
                                                      self.hdl.has_multicast_support) else 0
            self.peer_ptrs_dev = int(self.hdl.buffer_ptrs_dev)
            self.base_ptr = buf.data_ptr()
        # parameters in symmetric memory with an NVSwitch multicast mapping: the optimizer's
        # AdamW writes each updated bf16 value once for the whole group (the ZeRO parameter
        # all-gather fused into the step, ``adamw_all_gather``)
        self.pmc = 0
        if nvls:
            pbuf = symm_mem.empty(flat.numel, dtype=flat.data.dtype, device=dev)
            flat.rebind_data(pbuf)
            self.phdl = symm_mem.rendezvous(pbuf, group)
            if self.phdl.has_multicast_support:
                self.pmc = int(self.phdl.multicast_ptr)
        self.p_epoch = 0
        # the kernels' per-device status block (error word + wait limits)
        self.err = status_block(dev)
        self.epoch = 1
        torch.cuda.synchronize(dev)
        dist.barrier(group)

    @classmethod
    def create(cls, flat, group, use_multicast: bool = True, ring: bool = False
               ) -> "SymmReducer":
        return cls(flat, group, use_multicast, ring)

    def alloc_ring(self, n: int) -> torch.Tensor:
        """Symmetric fp32 buffer of the gradient ring (collective over the group)."""
        import torch.distributed._symmetric_memory as symm_mem
        buf = symm_mem.empty(n, dtype=torch.float32, device=self.device)
        self.rhdl = symm_mem.rendezvous(buf, self.group)
        self.mc = int(self.rhdl.multicast_ptr) if (self.use_multicast and
                                                   self.rhdl.has_multicast_support) else 0
        self.peer_ptrs_dev = int(self.rhdl.buffer_ptrs_dev)
        self.base_ptr = buf.data_ptr()
        self._ring_buf = buf
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)
        return buf

    @property
    def _pulled_base(self) -> int:
        return MAX_BUCKETS * self.W + 2 * self.W

    def slot_reuse_wait(self, idx: int):
        """Callable that orders the reuse of the ring slot of bucket ``idx`` (on the calling
        stream) after every peer has pulled that bucket of this micro-batch."""
        if not self.ring:
            return None
        epoch = self.epoch
        k = kernels()

        def wait():
            k.symm_wait(self.flags.data_ptr(), self._pulled_base + idx * self.W, 1, self.W,
                        epoch, self.err)
        return wait

    @property
    def kind(self) -> str:
        return "nvls-multimem" if self.mc else "p2p-loads"

    def reduce_bucket(self, idx: int, b, src: torch.Tensor, dst: torch.Tensor) -> None:
        assert idx < MAX_BUCKETS
        k = kernels()
        k.symm_signal(self.peer_flags_dev, self.W, idx * self.W + self.rank, self.epoch)
        k.symm_wait(self.flags.data_ptr(), idx * self.W, 1, self.W, self.epoch, self.err)
        off = (src.data_ptr() - self.base_ptr) // 4 + self.rank * b.chunk
        k.symm_pull_reduce(self.mc, self.peer_ptrs_dev, self.W, off, b.chunk, dst, 1.0, self.err)
        if self.ring:  # this rank has read every peer's slot of bucket idx
            k.symm_signal(self.peer_flags_dev, self.W,
                          self._pulled_base + idx * self.W + self.rank, self.epoch)

    def end_micro(self, flat) -> None:
        if self.ring:  # slots are protected per bucket by the pulled flags
            self.epoch += 1
            return
        k = kernels()
        base = MAX_BUCKETS * self.W
        k.symm_signal(self.peer_flags_dev, self.W, base + self.rank, self.epoch)
        k.symm_wait(self.flags.data_ptr(), base, 1, self.W, self.epoch, self.err)
        k.zero_unless_error(flat.grad, self.err)
        self.epoch += 1

    def adamw_all_gather(self, opt, coef: torch.Tensor) -> None:
        """AdamW on this rank's shard, bucket by bucket, with every updated bf16 parameter
        stored through the multicast address (all ranks receive it); then a bounded flag
        exchange orders the new parameters before anybody's next forward."""
        k = kernels()
        b1, b2 = opt.betas
        bc1 = 1.0 - b1 ** opt.step_count
        bc2 = 1.0 - b2 ** opt.step_count
        for b in opt.buckets:
            lo, hi = b.shard_off, b.shard_off + b.chunk
            k.adamw_multicast(opt.master[lo:hi], opt.grad_shard[lo:hi], opt.m[lo:hi],
                              opt.v[lo:hi], self.pmc + b.own_lo * 2, opt.lr, b1, b2, opt.eps,
                              opt.wd, bc1, bc2, coef)
        self.p_epoch += 1
        base = MAX_BUCKETS * self.W + self.W
        k.symm_signal(self.peer_flags_dev, self.W, base + self.rank, self.p_epoch)
        k.symm_wait(self.flags.data_ptr(), base, 1, self.W, self.p_epoch, self.err)

    def all_gather(self, dst: torch.Tensor, src_chunk: torch.Tensor) -> None:
        dist.all_gather_into_tensor(dst, src_chunk, group=self.group)

    def check(self) -> None:
        """Raise if a peer wait timed out (reads the device error word: host sync)."""
        v = int(self.err[0].item())
        if v:
            from ..utils.device_status import DeviceError
            self.err[:1].zero_()
            raise DeviceError(v)
