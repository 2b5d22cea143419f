"""Flat parameter / gradient storage.

All parameters of a model (or of one pipeline stage / tensor-parallel shard) live in ONE
contiguous bf16 buffer, and their gradients in ONE contiguous fp32 buffer with the same layout.
Every view starts on a 128-byte boundary (TMA needs 16-byte aligned bases and strides).

This layout is what the B200 data-parallel path is built around: ZeRO partitions are plain
slices of the flat buffers, reduce-scatter buckets are contiguous ranges, and the fused AdamW is
one kernel over a slice.  Parameters are laid out in the order in which the backward pass
finishes their gradients, last layer first, so buckets complete front to back.
"""
from __future__ import annotations

from collections import OrderedDict
from typing import Dict, Iterable, List, Tuple

import torch

ALIGN_ELEMS = 64  # 128 bytes of bf16


def _round_up(n: int, a: int) -> int:
    return (n + a - 1) // a * a


class FlatParams:
    """``bucket_numel`` (with ``pad_to`` = data-parallel size > 1) cuts the layout into buckets
    of about that many elements that never split a parameter, each padded to a multiple of
    ``pad_to * ALIGN_ELEMS`` (``bucket_bounds``): the units of the ZeRO reduce-scatter, and of
    the gradient ring of partitioned ZeRO-2 (a parameter's gradient must lie in one slot)."""

    def __init__(self, specs: Iterable[Tuple[str, Tuple[int, ...]]], device, pad_to: int = 1,
                 dtype=torch.bfloat16, grad_dtype=torch.float32, bucket_numel: int = 0):
        self.specs: "OrderedDict[str, Tuple[int, ...]]" = OrderedDict()
        self.offsets: Dict[str, int] = {}
        self.bucket_bounds: List[Tuple[int, int]] = []
        quantum = max(1, pad_to) * ALIGN_ELEMS
        bucketed = bucket_numel > 0 and pad_to > 1
        off = 0
        blo = 0
        for name, shape in specs:
            self.specs[name] = tuple(shape)
            n = 1
            for d in shape:
                n *= d
            if bucketed and off > blo and off + n - blo > bucket_numel:
                off = _round_up(off, quantum)
                self.bucket_bounds.append((blo, off))
                blo = off
            self.offsets[name] = off
            off = _round_up(off + n, ALIGN_ELEMS)
        self.numel = _round_up(off, quantum)
        if bucketed:
            self.bucket_bounds.append((blo, self.numel))
        self.device = torch.device(device)
        self.data = torch.zeros(self.numel, dtype=dtype, device=self.device)
        self.grad = torch.zeros(self.numel, dtype=grad_dtype, device=self.device)
        self.params: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        self.grads: "OrderedDict[str, torch.Tensor]" = OrderedDict()
        for name, shape in self.specs.items():
            o = self.offsets[name]
            n = 1
            for d in shape:
                n *= d
            self.params[name] = self.data[o:o + n].view(shape)
            self.grads[name] = self.grad[o:o + n].view(shape)

    def rebind_grad(self, buf: torch.Tensor) -> None:
        """Move the gradient storage to ``buf`` (e.g. symmetric memory for peer access)."""
        assert buf.numel() == self.numel and buf.dtype == self.grad.dtype
        buf.copy_(self.grad)
        self.grad = buf
        for name, shape in self.specs.items():
            o = self.offsets[name]
            n = 1
            for d in shape:
                n *= d
            self.grads[name] = self.grad[o:o + n].view(shape)

    def rebind_data(self, buf: torch.Tensor) -> None:
        """Move the parameter storage to ``buf`` (e.g. symmetric memory, so that the optimizer
        can write every rank's copy); parameter views are re-created."""
        assert buf.numel() == self.numel and buf.dtype == self.data.dtype
        buf.copy_(self.data)
        self.data = buf
        for name, shape in self.specs.items():
            o = self.offsets[name]
            n = 1
            for d in shape:
                n *= d
            self.params[name] = self.data[o:o + n].view(shape)

    def use_grad_ring(self, ring) -> None:
        """Partitioned gradients: ``grads[name]`` becomes a view into the ring slot that holds
        the parameter's bucket in the current micro-batch (acquired on first access), and the
        full-size ``grad`` buffer is released."""
        self.grad = None
        self.grads = _RingGradViews(self, ring)

    def names(self) -> List[str]:
        return list(self.specs)

    def zero_grad(self) -> None:
        self.grad.zero_()

    def range_of(self, name: str) -> Tuple[int, int]:
        o = self.offsets[name]
        n = 1
        for d in self.specs[name]:
            n *= d
        return o, o + n

    def __getitem__(self, name: str) -> torch.Tensor:
        return self.params[name]


class _RingGradViews:
    """Mapping name -> gradient view of :meth:`FlatParams.use_grad_ring` (see there)."""

    def __init__(self, flat: FlatParams, ring):
        self.flat, self.ring = flat, ring
        self.bucket_of: Dict[str, int] = {}
        for name in flat.specs:
            o = flat.offsets[name]
            for i, (lo, hi) in enumerate(flat.bucket_bounds):
                if lo <= o < hi:
                    self.bucket_of[name] = i
                    break

    def __getitem__(self, name: str) -> torch.Tensor:
        b = self.bucket_of[name]
        lo = self.flat.bucket_bounds[b][0]
        slot = self.ring.slot(b)
        o = self.flat.offsets[name] - lo
        shape = self.flat.specs[name]
        n = 1
        for d in shape:
            n *= d
        return slot[o:o + n].view(shape)

    def __iter__(self):
        return iter(self.flat.specs)

    def __len__(self) -> int:
        return len(self.flat.specs)

    def __contains__(self, name) -> bool:
        return name in self.flat.specs

    def keys(self):
        return self.flat.specs.keys()

    def items(self):
        return [(n, self[n]) for n in self.flat.specs]
