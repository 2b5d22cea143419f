"""Filtered training step on the native B200 models.

Per micro-batch: forward (fused lm_head + per-token CE), utility-based token selection
(``token_filter_loss``), ``backward_filter`` on the loss, the filtered backward (gradients
reduced on the fly by the ZeRO optimizer), and after ``grad_accum`` micro-batches one fused
AdamW step.  Mirrors ``Trainer.train_step`` of the reference (train.py:222-326) without its
host synchronisations: the only device-to-host reads are the optional loss readout and the
asynchronous copy of the kernels' status word, checked one step late.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .data.synthetic import Batch
from .filter import backward_filter
from .loss import keep_count, token_filter_loss


class Trainer:
    def __init__(self, model, optimizer, drop_rate: float = 0.5, strategy: str = "fixed",
                 grad_accum: int = 1, world_size: int = 1, timer=None,
                 filter_backward: bool = True, check_device_errors: bool = True):
        self.model = model
        self.opt = optimizer
        self.drop_rate = drop_rate
        self.strategy = strategy
        self.grad_accum = grad_accum
        self.world = world_size
        self.timer = timer
        # False = "loss only": the selection masks the loss but the backward stays dense
        self.filter_backward = filter_backward
        self.device = model.device
        if hasattr(optimizer, "attach"):
            optimizer.attach(model)
        # Device errors (a bounded wait that ran out, a mask row with the wrong keep count) are
        # read one step late from the kernels' status block; the failed step's AdamW update is
        # already skipped on the device.  Raises DeviceError.
        self.status = None
        if check_device_errors and torch.device(self.device).type == "cuda":
            from .utils.device_status import DeviceStatus
            self.status = DeviceStatus(self.device)

    def micro_step(self, batch: Batch, last: bool = True) -> torch.Tensor:
        """Forward + filtered backward of one micro-batch; ``last`` marks the last micro-batch
        before the optimizer step (the data-parallel gradient reduction runs in its backward)."""
        ids = batch.input_ids
        B, S = ids.shape
        out = self.model(ids)
        mask = (batch.attention_mask.clone() if batch.attention_mask is not None else
                torch.ones(B, S, dtype=torch.long, device=ids.device))
        if self.drop_rate > 0:
            loss, mask = token_filter_loss(ids, None, mask, batch.ref_loss, self.strategy,
                                           self.drop_rate, True, True,
                                           per_token_loss=out.token_loss)
            if self.strategy == "fixed" and batch.attention_mask is None:
                mask._cf_keep = keep_count(S, self.drop_rate)
            if self.filter_backward:
                backward_filter(loss, mask)
        else:
            loss = token_filter_loss(ids, None, mask, None, None, None, True,
                                     per_token_loss=out.token_loss)
        if hasattr(self.opt, "begin_micro"):
            self.opt.begin_micro(last=last)
        loss.backward()
        if hasattr(self.opt, "end_micro"):
            self.opt.end_micro()
        return loss.detach()

    def train_step(self, batches: Sequence[Batch], to_device: bool = True) -> torch.Tensor:
        """One optimizer step over ``grad_accum`` micro-batches; returns the mean loss (device)."""
        assert len(batches) == self.grad_accum
        total = torch.zeros((), device=self.device)
        for i, b in enumerate(batches):
            if to_device:
                b = b.to(self.device, non_blocking=True)
            total += self.micro_step(b, last=(i == len(batches) - 1))
        self.opt.step(grad_scale=1.0 / (self.grad_accum * self.world))
        self.opt.zero_grad()
        if self.status is not None:
            self.status.record()
        return total / self.grad_accum
