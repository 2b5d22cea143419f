"""Device-side failure reporting for the training loop.

Every sm_100a kernel of this package receives the per-device status block (four int32 words,
``kernels().status_block(device)``): word 0 holds the first error code a kernel recorded, words 1
and 2 the limits of the bounded waits (microseconds; 0 = defaults of 4 s on the GPU's own work and
20 s on another GPU).  A wait that runs out records its code and returns; the kernels that follow
in the same step see the word set and skip what would consume half-finished data (the NVLink
gradient pull, the clearing of a gradient buffer a peer may still read, the AdamW update).

:class:`DeviceStatus` brings the word to the host without stalling the GPU: at the end of step n
it queues an asynchronous copy of the block into pinned memory and checks the copy of step n-1,
which has completed by then (one step of lag, the GPU always has a full step queued).  A set word
raises :class:`DeviceError` -- the reference skips a step whose filter raised (train.py:261-269);
here the step's update is already skipped on the device, and the host learns of it one step late.
"""
from __future__ import annotations

from typing import Optional

import torch

ERROR_CODES = {
    1: "a TMA producer wait ran out",
    2: "an MMA-issuer wait ran out",
    3: "an epilogue wait ran out",
    4: "a softmax-warp wait ran out",
    16: "a kernel rejected its arguments",
    32: "a wait on another GPU ran out (peer flag not raised in time)",
    64: "a mask row did not keep the expected number of tokens",
    128: "an index (token id, label or row id) was outside its table; the access was skipped",
}


def describe(code: int) -> str:
    return ERROR_CODES.get(int(code), f"unknown device error code {int(code)}")


class DeviceError(RuntimeError):
    def __init__(self, code: int, step: Optional[int] = None):
        self.code = int(code)
        self.step = step
        where = f" in step {step}" if step is not None else ""
        super().__init__(f"device error{where}: {describe(code)} (code {self.code})")


class DeviceStatus:
    """Reads a status block one step late.

    ``block`` defaults to the kernels' status block of ``device``; tests may pass any int32
    tensor of at least one word (a CPU tensor is read synchronously).
    """

    def __init__(self, device, block: Optional[torch.Tensor] = None):
        self.device = torch.device(device)
        if block is None:
            from ..ops._ext import status_block
            block = status_block(self.device)
        self.block = block
        self.async_copy = block.is_cuda
        self.host = torch.zeros(2, block.numel(), dtype=torch.int32,
                                pin_memory=self.async_copy)
        self._events = [None, None]
        self._steps = [None, None]
        self.step = 0

    def set_wait_limits(self, local_s: float = 0.0, peer_s: float = 0.0) -> None:
        """Limits of the bounded device waits (seconds; 0 = default)."""
        from ..ops._ext import kernels
        idx = self.device.index if self.device.index is not None else torch.cuda.current_device()
        kernels().set_wait_limits(idx, int(local_s * 1e6), int(peer_s * 1e6))

    def _check_row(self, slot: int) -> None:
        code = int(self.host[slot, 0])
        if code:
            step = self._steps[slot]
            self.block[:1].zero_()  # the caller may continue after handling the error
            # copies queued before this reset still hold the same error: drop them
            self._events = [None, None]
            raise DeviceError(code, step)

    def record(self) -> None:
        """End of a step: queue the copy of this step's word, check the previous step's."""
        slot = self.step % 2
        if self._events[slot] is not None:  # two steps old (only if record was skipped)
            self._events[slot].synchronize()
            self._events[slot] = None
            self._check_row(slot)
        self.host[slot].copy_(self.block, non_blocking=self.async_copy)
        self._steps[slot] = self.step
        if self.async_copy:
            ev = torch.cuda.Event()
            ev.record()
            self._events[slot] = ev
        else:
            self._events[slot] = None
            self.step += 1
            self._check_row(slot)
            return
        self.step += 1
        prev = 1 - slot
        if self._events[prev] is not None:
            self._events[prev].synchronize()
            self._events[prev] = None
            self._check_row(prev)

    def check_now(self) -> None:
        """Wait for all queued work and raise if any step recorded an error."""
        for slot in (0, 1):
            if self._events[slot] is not None:
                self._events[slot].synchronize()
                self._events[slot] = None
                self._check_row(slot)
        if self.async_copy:
            torch.cuda.synchronize(self.device)
        self.host[0].copy_(self.block)
        self._steps[0] = self.step
        self._check_row(0)
