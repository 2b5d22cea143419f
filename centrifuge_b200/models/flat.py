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
    def __init__(self, specs: Iterable[Tuple[str, Tuple[int, ...]]], device, pad_to: int = 1,
                 dtype=torch.bfloat16, grad_dtype=torch.float32):
        self.specs: "OrderedDict[str, Tuple[int, ...]]" = OrderedDict()
        self.offsets: Dict[str, int] = {}
        off = 0
        for name, shape in specs:
            self.specs[name] = tuple(shape)
            self.offsets[name] = off
            n = 1
            for d in shape:
                n *= d
            off = _round_up(off + n, ALIGN_ELEMS)
        self.numel = _round_up(off, max(1, pad_to) * ALIGN_ELEMS)
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
