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
    def __init__(self, flat, group, use_multicast: bool = True):
        import torch.distributed._symmetric_memory as symm_mem
        self.group = group
        self.W = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        dev = flat.device
        buf = symm_mem.empty(flat.numel, dtype=torch.float32, device=dev)
        flat.rebind_grad(buf)
        self.flat = flat
        self.hdl = symm_mem.rendezvous(buf, group)
        self.mc = int(self.hdl.multicast_ptr) if (use_multicast and
                                                  self.hdl.has_multicast_support) else 0
        self.peer_ptrs_dev = int(self.hdl.buffer_ptrs_dev)
        # parameters in symmetric memory with an NVSwitch multicast mapping: the optimizer's
        # AdamW writes each updated bf16 value once for the whole group (the ZeRO parameter
        # all-gather fused into the step, ``adamw_all_gather``)
        self.pmc = 0
        if self.mc:
            pbuf = symm_mem.empty(flat.numel, dtype=flat.data.dtype, device=dev)
            flat.rebind_data(pbuf)
            self.phdl = symm_mem.rendezvous(pbuf, group)
            if self.phdl.has_multicast_support:
                self.pmc = int(self.phdl.multicast_ptr)
        self.p_epoch = 0
        nflags = MAX_BUCKETS * self.W + 2 * self.W
        self.flags = symm_mem.empty(nflags, dtype=torch.int32, device=dev)
        self.flags.zero_()
        self.fhdl = symm_mem.rendezvous(self.flags, group)
        self.peer_flags_dev = int(self.fhdl.buffer_ptrs_dev)
        # the kernels' per-device status block (error word + wait limits)
        self.err = status_block(dev)
        self.epoch = 1
        self.base_ptr = buf.data_ptr()
        torch.cuda.synchronize(dev)
        dist.barrier(group)

    @classmethod
    def create(cls, flat, group, use_multicast: bool = True) -> "SymmReducer":
        return cls(flat, group, use_multicast)

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

    def end_micro(self, flat) -> None:
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
