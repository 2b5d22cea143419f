"""ZeRO-1 / ZeRO-2 data parallelism with a fused AdamW over a flat parameter buffer.

Reference behaviour: DeepSpeed ZeRO stage 1 with AdamW, gradient clipping 1.0, bf16, 2e8-element
reduce-scatter / all-gather buckets and ``overlap_comm`` (train.py:109-157).  Stage 2 (gradient
partitioning during the backward) is what the B200 workload uses.

Layout.  The model's parameters live in one flat buffer (:class:`~centrifuge_b200.models.flat.
FlatParams`), laid out so that gradients complete front to back during the backward.  The flat
range is cut into buckets; rank ``r`` owns chunk ``r`` of every bucket ("bucket-major"
sharding), so a bucket is reduce-scattered as soon as the backward has finished it and each
rank's optimizer shard is the concatenation of its chunks.

Stage 2 has two gradient modes.

* ``grad_mode="ring"`` (partitioned, DeepSpeed ZeRO-2 semantics): no full-size gradient buffer.
  The layout is cut into buckets that never split a parameter (``FlatParams.bucket_bounds``); a
  bucket's gradients are written into one of ``ring_slots`` bucket-sized fp32 slots
  (:class:`GradRing`), and as soon as the backward has finished the bucket it is reduce-scattered
  into the rank's fp32 gradient shard, in every micro-batch.  A slot is reused only after its
  reduction (and, over NVLink, every peer's read of it) has completed.  Gradient memory per rank
  is the shard (1/W) plus ``ring_slots`` buckets.
* ``grad_mode="full"`` (local accumulation, one reduction per step): every rank keeps a
  full-size fp32 gradient buffer; the micro-batches of a step accumulate into it and the buckets
  are reduced during the backward of the last micro-batch only, so a step moves each gradient
  over NVLink once instead of ``grad_accum`` times.  Its gradient memory is that of ZeRO-1.
  ``reduce_every_micro=True`` reduces in every micro-batch instead.

Stage 1 accumulates the full local gradients over the micro-batches and reduces once at the
boundary, without overlap.

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


def _buckets_per_unit(flat) -> int:
    """Largest number of buckets whose gradients a model writes before it reports any of them
    final: the parameters of one layer ("layers.<i>.*"), of the head (lm_head + norm), or the
    embedding.  The gradient ring needs one slot more than that."""
    units = {}
    for name in flat.specs:
        if name.startswith("layers."):
            key = name.rsplit(".", 1)[0]
        else:
            key = "head" if name in ("lm_head", "norm") else name
        o = flat.offsets[name]
        for i, (lo, hi) in enumerate(flat.bucket_bounds):
            if lo <= o < hi:
                units.setdefault(key, set()).add(i)
                break
    return max((len(v) for v in units.values()), default=1)


def _world(group):
    """(size, rank) of the data-parallel group; ``None`` means no data parallelism."""
    if group is None:
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


class GradRing:
    """Bucket-sized fp32 gradient slots of partitioned ZeRO-2.

    Bucket ``b`` uses slot ``b % slots``.  :meth:`slot` hands out the bucket's slot on the
    first access of a micro-batch, after running the ordering callable left by the slot's
    previous bucket; :meth:`released` records that callable when the reduction of a bucket has
    been issued.  Slots start zeroed and are cleared again on the communication stream right
    after their reduction (once every reader is done), so the backward finds them zero without
    a memset of its own.  A bucket that needs a slot whose previous bucket is not reduced yet
    raises: the layer being differentiated spans more buckets than there are slots.
    """

    def __init__(self, buckets, slots: int, device, alloc=None):
        self.sizes = [b.hi - b.lo for b in buckets]
        self.slot_numel = max(self.sizes)
        self.R = max(1, min(slots, len(buckets)))
        n = self.R * self.slot_numel
        self.buf = (alloc(n) if alloc is not None
                    else torch.empty(n, dtype=torch.float32, device=device))
        self.buf.zero_()
        self.cur = {}
        self.holder = [None] * self.R
        self.pending = [False] * self.R
        self.before_reuse = [None] * self.R

    @property
    def nbytes(self) -> int:
        return self.buf.numel() * self.buf.element_size()

    def begin_micro(self) -> None:
        self.cur = {}

    def _view(self, s: int, b: int) -> torch.Tensor:
        return self.buf[s * self.slot_numel:s * self.slot_numel + self.sizes[b]]

    def slot(self, b: int) -> torch.Tensor:
        s = self.cur.get(b)
        if s is None:
            s = b % self.R
            if self.pending[s]:
                raise RuntimeError(
                    f"gradient ring: bucket {b} needs slot {s}, which still holds bucket "
                    f"{self.holder[s]} (not reduced yet); use more ring slots")
            if self.before_reuse[s] is not None:
                self.before_reuse[s]()
                self.before_reuse[s] = None
            self.cur[b] = s
            self.holder[s] = b
            self.pending[s] = True
        return self._view(s, b)

    def released(self, b: int, before_reuse) -> None:
        s = self.cur[b]
        self.pending[s] = False
        self.before_reuse[s] = before_reuse


class NcclReducer:
    """Reduce-scatter baseline: cast the bucket to ``comm_dtype``, NCCL reduce-scatter, add the
    result to the fp32 shard."""

    def __init__(self, group, comm_dtype=torch.bfloat16):
        self.group = group
        self.comm_dtype = comm_dtype
        self._send = None
        self._recv = None
        self.ring = False  # partitioned gradients: the slot is cleared on its next use instead

    def reduce_bucket(self, idx: int, b, src_fp32: torch.Tensor, dst_fp32: torch.Tensor) -> None:
        self.reduce_scatter_acc(src_fp32, dst_fp32, 1.0)
        if not self.ring:
            src_fp32.zero_()

    def slot_reuse_wait(self, idx: int):
        """Extra ordering before a ring slot that held bucket ``idx`` is written again (none:
        the NCCL reduction is ordered by the communication stream's event)."""
        return None

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
                 replication: Optional[int] = None, reduce_every_micro: bool = False,
                 grad_mode: str = "full", ring_slots: int = 4):
        assert stage in (1, 2)
        assert grad_mode in ("full", "ring")
        self.W, self.rank = _world(group)
        # partitioned gradients need more than one rank and the bucket-aligned layout
        self.grad_mode = grad_mode if (stage == 2 and self.W > 1 and flat.bucket_bounds) else "full"
        if grad_mode == "ring" and self.grad_mode != "ring" and self.W > 1:
            raise ValueError("grad_mode='ring' needs stage 2 and a FlatParams built with "
                             "bucket_numel (pad_to = data-parallel size)")
        self.reduce_every_micro = reduce_every_micro or self.grad_mode == "ring"
        self._active = True  # this micro-batch's backward reduces buckets
        self.flat = flat
        self.group = group
        self.stage = stage
        self.lr, self.betas, self.eps, self.wd = lr, tuple(betas), eps, weight_decay
        self.grad_clip = grad_clip
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
        bounds = list(flat.bucket_bounds) if (flat.bucket_bounds and self.W > 1) else None
        while lo < N:
            hi = bounds[len(self.buckets)][1] if bounds else min(N, lo + bucket_numel)
            assert (hi - lo) % quantum == 0, "bucket not divisible into aligned rank chunks"
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
        self.ring = None
        if self.grad_mode == "ring":
            self.reducer.ring = True
            slots = max(ring_slots, _buckets_per_unit(flat) + 1)
            self.ring = GradRing(self.buckets, slots, self.device,
                                 alloc=getattr(self.reducer, "alloc_ring", None))
            flat.use_grad_ring(self.ring)
        self._coef = torch.ones(1, **f32)
        self._norm = torch.zeros(1, **f32)
        self._sumsq = torch.zeros(148 * 4, **f32)
        self._sumsq_total = torch.zeros(1, **f32)
        self._comm_stream = torch.cuda.Stream(device=self.device) if self.overlap else None
        self._ready = 0  # buckets reduced in the current micro-batch
        self._last = True  # the current micro-batch is the last before step()
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
        self._last = last
        self._active = last or self.reduce_every_micro
        if self.ring is not None:
            self.ring.begin_micro()

    def on_grads_ready(self, lo: int, hi: int) -> None:
        if not self._active:
            return  # gradients keep accumulating in the local buffer
        # gradients complete front to back: every bucket ending at or before `hi` is final
        while self._ready < len(self.buckets) and self.buckets[self._ready].hi <= hi:
            self._reduce_bucket(self.buckets[self._ready])
            self._ready += 1

    def _reduce_bucket(self, b: Bucket) -> None:
        idx = self.buckets.index(b) if not hasattr(b, "idx") else b.idx
        # a bucket without gradients in this micro-batch still takes part (zero slot)
        src = self.ring.slot(idx) if self.ring is not None else self.flat.grad[b.lo:b.hi]
        dst = self.grad_shard[b.shard_off:b.shard_off + b.chunk]
        ev = None

        def reduce_and_clear():
            self.reducer.reduce_bucket(idx, b, src, dst)
            if self.ring is not None:
                # clear the slot for its next bucket once every reader (over NVLink: every
                # peer) is done with it, off the backward's stream
                peers = self.reducer.slot_reuse_wait(idx)
                if peers is not None:
                    peers()
                src.zero_()

        if self._comm_stream is not None:
            cur = torch.cuda.current_stream(self.device)
            self._comm_stream.wait_stream(cur)
            with torch.cuda.stream(self._comm_stream):
                reduce_and_clear()
                if self.ring is not None:
                    ev = torch.cuda.Event()
                    ev.record()
        else:
            reduce_and_clear()
        if self.ring is not None:
            dev = self.device

            def before_reuse(ev=ev):
                if ev is not None:
                    torch.cuda.current_stream(dev).wait_event(ev)

            self.ring.released(idx, before_reuse)

    def end_micro(self) -> None:
        """Finish the micro-batch: reduce what is left (stage 2) and join the comm stream."""
        if self.W == 1 or not self._active:
            return
        if self.stage == 2:
            self.on_grads_ready(0, self.flat.numel)
            self._finish_reducer()
        if self._comm_stream is not None and (self._last or self.ring is None):
            # The next micro-batch's forward touches neither the ring nor the shard: with
            # partitioned gradients the tail of this micro-batch's reductions (the first
            # layers and the embedding) keeps running under it.  Ring slots are ordered by
            # their own events, the optimizer step joins after the last micro-batch.
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

    def grad_memory_bytes(self) -> int:
        """Device bytes held for gradients on this rank (local buffer or ring + fp32 shard)."""
        shard = 0 if self.W == 1 else self.grad_shard.numel() * 4
        if self.ring is not None:
            return self.ring.nbytes + shard
        return self.flat.grad.numel() * self.flat.grad.element_size() + shard

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
