"""ZeRO-1 / ZeRO-2 data parallelism with a fused AdamW over a flat parameter buffer.

Reference behaviour: DeepSpeed ZeRO stage 1 with AdamW, gradient clipping 1.0, bf16, 2e8-element
reduce-scatter / all-gather buckets and ``overlap_comm`` (train.py:109-157).  Stage 2 (gradient
partitioning during the backward) is what the B200 workload uses.

Layout.  The model's parameters live in one flat buffer (:class:`~centrifuge_b200.models.flat.
FlatParams`), laid out so that gradients complete front to back during the backward.  The flat
range is cut into buckets; rank ``r`` owns chunk ``r`` of every bucket ("bucket-major"
sharding), so a bucket is reduce-scattered as soon as the backward has finished it and each
rank's optimizer shard is the concatenation of its chunks.

Stage 2: when a bucket's gradients are final the bucket is reduced on a communication stream
into the rank's fp32 gradient shard and its slice of the local gradient buffer is cleared.  By
default this happens only in the backward of the last micro-batch of a step: the earlier
micro-batches accumulate into the local fp32 buffer (which is full-size here anyway), so a step
moves each gradient over NVLink once instead of ``grad_accum`` times, and the reduction still
overlaps the last backward bucket by bucket.  ``reduce_every_micro=True`` reduces in every
micro-batch's backward, as DeepSpeed's ZeRO-2 does.  Stage 1 accumulates the full local
gradients over the micro-batches and reduces once at the boundary, without overlap.

Step: global grad-norm (local sum of squares + one 4-byte all-reduce), clip coefficient computed
on the device, fused AdamW on the fp32 master shard writing bf16 parameters, then a per-bucket
all-gather of the parameters.  No host synchronisation anywhere on this path.

The reduction itself is pluggable (``reducer``): :class:`NcclReducer` is the NCCL baseline
(bf16 on the wire, fp32 accumulate); :mod:`centrifuge_b200.parallel.symm` provides the fused
sm_100a kernel over NVLink peer memory.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from ..models.flat import ALIGN_ELEMS, FlatParams
from ..ops import fused


@dataclass
class Bucket:
    lo: int  # flat range [lo, hi)
    hi: int
    chunk: int  # elements per rank
    shard_off: int  # offset of this rank's chunk inside the shard buffers

    @property
    def own_lo(self) -> int:  # set by the optimizer
        return self._own_lo


def _world(group):
    """(size, rank) of the data-parallel group; ``None`` means no data parallelism."""
    if group is None:
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


class NcclReducer:
    """Reduce-scatter baseline: cast the bucket to ``comm_dtype``, NCCL reduce-scatter, add the
    result to the fp32 shard."""

    def __init__(self, group, comm_dtype=torch.bfloat16):
        self.group = group
        self.comm_dtype = comm_dtype
        self._send = None
        self._recv = None

    def reduce_bucket(self, idx: int, b, src_fp32: torch.Tensor, dst_fp32: torch.Tensor) -> None:
        self.reduce_scatter_acc(src_fp32, dst_fp32, 1.0)
        src_fp32.zero_()

    def end_micro(self, flat) -> None:
        pass

    def reduce_scatter_acc(self, src_fp32: torch.Tensor, dst_fp32: torch.Tensor, scale: float):
        n, c = src_fp32.numel(), dst_fp32.numel()
        if self._send is None or self._send.numel() < n:
            self._send = torch.empty(n, dtype=self.comm_dtype, device=src_fp32.device)
            self._recv = torch.empty(c, dtype=self.comm_dtype, device=src_fp32.device)
        send, recv = self._send[:n], self._recv[:c]
        if self.comm_dtype == torch.float32:
            send = src_fp32
            recv = torch.empty_like(dst_fp32)
        else:
            send.copy_(src_fp32)
        dist.reduce_scatter_tensor(recv, send, group=self.group)
        dst_fp32.add_(recv.float() if recv.dtype != torch.float32 else recv, alpha=scale)

    def all_gather(self, dst: torch.Tensor, src_chunk: torch.Tensor):
        dist.all_gather_into_tensor(dst, src_chunk, group=self.group)


class ZeroAdamW:
    def __init__(self, flat: FlatParams, group=None, stage: int = 2, lr: float = 1e-4,
                 betas=(0.9, 0.95), eps: float = 1e-8, weight_decay: float = 0.0,
                 grad_clip: float = 1.0, bucket_numel: int = 1 << 26, reducer=None,
                 overlap: bool = True, norm_group=None, replicated_ranges=(),
                 replication: Optional[int] = None, reduce_every_micro: bool = False):
        assert stage in (1, 2)
        self.reduce_every_micro = reduce_every_micro
        self._active = True  # this micro-batch's backward reduces buckets
        self.flat = flat
        self.group = group
        self.stage = stage
        self.lr, self.betas, self.eps, self.wd = lr, tuple(betas), eps, weight_decay
        self.grad_clip = grad_clip
        self.W, self.rank = _world(group)
        self.device = flat.device
        self.step_count = 0
        self.overlap = overlap and self.W > 1 and flat.device.type == "cuda"
        quantum = self.W * ALIGN_ELEMS
        N = flat.numel
        assert N % quantum == 0, f"flat buffer ({N}) must be padded to a multiple of {quantum}"
        bucket_numel = max(quantum, bucket_numel // quantum * quantum)
        self.buckets: List[Bucket] = []
        off = 0
        lo = 0
        while lo < N:
            hi = min(N, lo + bucket_numel)
            chunk = (hi - lo) // self.W
            b = Bucket(lo, hi, chunk, off)
            b._own_lo = lo + self.rank * chunk
            b.idx = len(self.buckets)
            self.buckets.append(b)
            off += chunk
            lo = hi
        self.shard_numel = off
        f32 = dict(dtype=torch.float32, device=self.device)
        # fp32 master copy of the owned parameters (bucket-major order)
        self.master = torch.empty(self.shard_numel, **f32)
        for b in self.buckets:
            self.master[b.shard_off:b.shard_off + b.chunk].copy_(flat.data[b.own_lo:b.own_lo + b.chunk])
        self.m = torch.zeros(self.shard_numel, **f32)
        self.v = torch.zeros(self.shard_numel, **f32)
        if self.W == 1:
            self.grad_shard = flat.grad  # no partitioning on one rank
            self.param_out = flat.data
        else:
            self.grad_shard = torch.zeros(self.shard_numel, **f32)
            self.param_out = torch.empty(self.shard_numel, dtype=flat.data.dtype, device=self.device)
        self.reducer = reducer if reducer is not None else (
            NcclReducer(group) if self.W > 1 else None)
        self._coef = torch.ones(1, **f32)
        self._norm = torch.zeros(1, **f32)
        self._sumsq = torch.zeros(148 * 4, **f32)
        self._sumsq_total = torch.zeros(1, **f32)
        self._comm_stream = torch.cuda.Stream(device=self.device) if self.overlap else None
        self._ready = 0  # buckets reduced in the current micro-batch
        self.grad_scale = 1.0
        # Model-parallel group whose ranks hold different shards of the model: the grad-norm
        # sums over it; ``replicated_ranges`` (flat [lo, hi) ranges of parameters replicated on
        # every rank of that group) are counted once.
        self.norm_group = norm_group
        self.norm_world = dist.get_world_size(norm_group) if norm_group is not None else 1
        self.replicated_ranges = list(replicated_ranges)
        self.replication = replication or self.norm_world
        if self.replicated_ranges and self.norm_world > 1:
            assert self.W == 1, "replicated-parameter norm correction needs data-parallel size 1"
        # callables run at the start of step(), e.g. summing replicated gradients over TP
        self.pre_step_hooks = []

    # ------------------------------------------------------------------ backward hooks
    def attach(self, model) -> None:
        """Reduce buckets as the model's backward finishes them (stage 2)."""
        if self.stage == 2 and self.W > 1:
            model.grad_ready_hook = self.on_grads_ready

    def begin_micro(self, last: bool = True) -> None:
        """Start a micro-batch; ``last`` marks the last one before :meth:`step`."""
        self._ready = 0
        self._active = last or self.reduce_every_micro

    def on_grads_ready(self, lo: int, hi: int) -> None:
        if not self._active:
            return  # gradients keep accumulating in the local buffer
        # gradients complete front to back: every bucket ending at or before `hi` is final
        while self._ready < len(self.buckets) and self.buckets[self._ready].hi <= hi:
            self._reduce_bucket(self.buckets[self._ready])
            self._ready += 1

    def _reduce_bucket(self, b: Bucket) -> None:
        src = self.flat.grad[b.lo:b.hi]
        dst = self.grad_shard[b.shard_off:b.shard_off + b.chunk]
        idx = self.buckets.index(b) if not hasattr(b, "idx") else b.idx
        if self._comm_stream is not None:
            cur = torch.cuda.current_stream(self.device)
            self._comm_stream.wait_stream(cur)
            with torch.cuda.stream(self._comm_stream):
                self.reducer.reduce_bucket(idx, b, src, dst)
        else:
            self.reducer.reduce_bucket(idx, b, src, dst)

    def end_micro(self) -> None:
        """Finish the micro-batch: reduce what is left (stage 2) and join the comm stream."""
        if self.W == 1 or not self._active:
            return
        if self.stage == 2:
            self.on_grads_ready(0, self.flat.numel)
            self._finish_reducer()
        if self._comm_stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._comm_stream)

    def _finish_reducer(self) -> None:
        if self._comm_stream is not None:
            with torch.cuda.stream(self._comm_stream):
                self.reducer.end_micro(self.flat)
        else:
            self.reducer.end_micro(self.flat)

    # ------------------------------------------------------------------ step
    def zero_grad(self) -> None:
        if self.W == 1:
            self.flat.grad.zero_()
        else:
            self.grad_shard.zero_()
            if self.stage == 1:
                self.flat.grad.zero_()

    def _reduce_all_stage1(self) -> None:
        for b in self.buckets:
            self._reduce_bucket(b)
        self._finish_reducer()
        if self._comm_stream is not None:
            torch.cuda.current_stream(self.device).wait_stream(self._comm_stream)

    def step(self, grad_scale: float = 1.0) -> torch.Tensor:
        """One optimizer step.  ``grad_scale`` multiplies the accumulated gradient sum (e.g.
        ``1 / (grad_accum * world)``).  Returns the (device) global grad-norm tensor."""
        if self.W > 1 and self.stage == 1:
            self._reduce_all_stage1()
        for hook in self.pre_step_hooks:
            hook()
        self.step_count += 1
        g = self.grad_shard
        if self.norm_world > 1:
            tot = g.float().pow(2).sum().view(1)
            if self.replicated_ranges:
                rep = sum(g[lo:hi].float().pow(2).sum() for lo, hi in self.replicated_ranges)
                tot = tot - (1.0 - 1.0 / self.replication) * rep
            self._sumsq_total.copy_(tot)
            if self.W > 1:
                dist.all_reduce(self._sumsq_total, group=self.group)
            dist.all_reduce(self._sumsq_total, group=self.norm_group)
            fused.grad_norm_clip_coef(g, self.grad_clip, grad_scale, self._coef, self._norm,
                                      extra_sumsq=self._sumsq_total)
        elif self.W > 1:
            if g.is_cuda:
                fused.kernels().sumsq(g, self._sumsq)
                torch.sum(self._sumsq, dim=0, keepdim=True, out=self._sumsq_total)
            else:
                self._sumsq_total.copy_(g.pow(2).sum().view(1))
            dist.all_reduce(self._sumsq_total, group=self.group)
            fused.grad_norm_clip_coef(g, self.grad_clip, grad_scale, self._coef, self._norm,
                                      extra_sumsq=self._sumsq_total)
        else:
            fused.grad_norm_clip_coef(g, self.grad_clip, grad_scale, self._coef, self._norm,
                                      partial=self._sumsq)
        coef = self._coef if g.is_cuda else float(self._coef.item())
        b1, b2 = self.betas
        if self.W > 1 and getattr(self.reducer, "pmc", 0):
            # parameter all-gather fused into AdamW (NVSwitch multicast stores)
            self.reducer.adamw_all_gather(self, coef)
            return self._norm
        fused.adamw_(self.master, g, self.m, self.v, self.param_out, self.lr, b1, b2, self.eps,
                     self.wd, self.step_count, coef)
        if self.W > 1:
            for b in self.buckets:
                self.reducer.all_gather(self.flat.data[b.lo:b.hi],
                                        self.param_out[b.shard_off:b.shard_off + b.chunk])
        return self._norm

    # ------------------------------------------------------------------ state
    def state_dict(self):
        return {"master": self.master, "m": self.m, "v": self.v,
                "step": torch.tensor(self.step_count)}

    def load_state_dict(self, sd) -> None:
        self.master.copy_(sd["master"])
        self.m.copy_(sd["m"])
        self.v.copy_(sd["v"])
        self.step_count = int(sd["step"])
        # re-materialise the bf16 parameters from the master shard
        if self.W == 1:
            self.flat.data.copy_(self.master)
        else:
            self.param_out.copy_(self.master)
            for b in self.buckets:
                self.reducer.all_gather(self.flat.data[b.lo:b.hi],
                                        self.param_out[b.shard_off:b.shard_off + b.chunk])
