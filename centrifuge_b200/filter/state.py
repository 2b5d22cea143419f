"""Kept-token state shared by the filtered backward nodes of one micro-batch.

A :class:`FilterState` is built once from the ``[B, S]`` keep mask (1 = keep):

* ``s_keep``      kept tokens per row (every row keeps the same count, as the reference
                  requires: graph_filter.cpp:48-50, backward_filters.cpp:204-208)
* ``pos``         ``[B, S_keep]`` int32 kept positions, ascending
* ``rows``        ``[B*S_keep]`` int32 flattened kept-row ids ``b*S + pos`` into ``[B*S, ...]``
* ``loss_rows``   ``[B*(S_keep-1)]`` kept rows of the ``[B, S-1]`` per-token loss

``S_keep`` is taken from the mask's ``_cf_keep`` attribute when the selection attached it
(``token_filter_loss`` knows ``S - k`` statically), so building the state needs no host
synchronisation.  Without it, one ``mask.sum()`` is read back, as the reference does.
"""
from __future__ import annotations

from typing import Optional

import torch


class FilterState:
    def __init__(self, mask: torch.Tensor, s_keep: Optional[int] = None):
        if mask.dim() != 2:
            raise ValueError(f"mask must be [B, S], got {tuple(mask.shape)}")
        self.B, self.S = int(mask.shape[0]), int(mask.shape[1])
        if s_keep is None:
            s_keep = getattr(mask, "_cf_keep", None)
        if s_keep is None:
            total = int(mask.sum().item())
            if total % self.B:
                raise ValueError("every row of the mask must keep the same number of tokens")
            s_keep = total // self.B
        self.s_keep = int(s_keep)
        from ..ops import select
        self.pos, self.rows, self.err = select.keep_index(mask, self.s_keep)
        self.pos_flat = self.pos.reshape(-1).contiguous()
        self.device = mask.device

    @property
    def t_keep(self) -> int:
        return self.B * self.s_keep

    def check(self):
        """Raise if a row did not keep ``s_keep`` tokens (host sync; used by tests/debug).

        On the GPU this reads the device status block, which also collects the other kernels'
        errors; the training loop reads it asynchronously instead (``DeviceStatus``)."""
        code = int(self.err.reshape(-1)[0].item())
        if code != 0:
            self.err.reshape(-1)[:1].zero_()
            raise ValueError(f"mask rows do not all keep {self.s_keep} tokens (device code {code})")


def state_for_mask(mask: torch.Tensor) -> FilterState:
    """One :class:`FilterState` per mask tensor object (shared by all nodes it filters).

    The state is cached on the tensor object and rebuilt if the mask was modified in place
    since (its version counter changed).
    """
    st = getattr(mask, "_cf_state", None)
    if st is None or st._version != mask._version:
        st = FilterState(mask)
        st._version = mask._version
        mask._cf_state = st
    return st


class FilterSlot:
    """Holder that a native backward node reads at backward time; empty = unfiltered."""

    __slots__ = ("state",)

    def __init__(self):
        self.state: Optional[FilterState] = None

    def attach(self, mask: torch.Tensor) -> None:
        self.state = state_for_mask(mask)
