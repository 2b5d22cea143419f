"""Per-phase step timing with CUDA events (no synchronisation inside the step).

Reference: ``BatchTimer`` (model/utils.py:12-73) takes wall-clock timestamps after explicit
``torch.cuda.synchronize()`` calls, pushes NVTX ranges and dumps per-step JSON with warm-up-
excluded averages.  Here phases are bracketed by CUDA events recorded on the current stream and
resolved only when the step is closed; NVTX ranges and the JSON dump are kept.
"""
from __future__ import annotations

import json
import time
from typing import Dict, List, Optional

import torch


class StepTimer:
    def __init__(self, output_file: Optional[str] = None, warmup: int = 2, nvtx: bool = True,
                 enabled: bool = True):
        self.output_file = output_file
        self.warmup = warmup
        self.nvtx = nvtx and torch.cuda.is_available()
        self.enabled = enabled and torch.cuda.is_available()
        self.steps: List[Dict[str, float]] = []
        self._events: List = []
        self._names: List[str] = []
        self._t0 = None
        self._step = 0

    def start(self):
        self._step += 1
        self._events, self._names = [], []
        self._t0 = time.perf_counter()
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events.append(e)
            self._names.append("start")
        if self.nvtx:
            torch.cuda.nvtx.range_push(f"step {self._step}")

    def record(self, name: str):
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self._events.append(e)
            self._names.append(name)
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
            torch.cuda.nvtx.range_push(name)

    def end(self) -> Dict[str, float]:
        rec: Dict[str, float] = {}
        if self.enabled:
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            e.synchronize()
            self._events.append(e)
            self._names.append("end")
            for i in range(1, len(self._events)):
                name = self._names[i] if self._names[i] != "end" else "tail"
                rec[name] = rec.get(name, 0.0) + self._events[i - 1].elapsed_time(self._events[i])
            rec["total"] = self._events[0].elapsed_time(self._events[-1])
        rec["wall_total"] = (time.perf_counter() - self._t0) * 1000.0
        if self.nvtx:
            torch.cuda.nvtx.range_pop()
        self.steps.append(rec)
        if self.output_file:
            self.dump()
        return rec

    def averages(self) -> Dict[str, float]:
        keys = set()
        for s in self.steps:
            keys |= set(s)
        out = {}
        tail = self.steps[self.warmup:]
        for k in keys:
            vals = [s[k] for s in tail if k in s]
            out[k + "_avg"] = sum(vals) / len(vals) if vals else 0.0
        return out

    def dump(self):
        with open(self.output_file, "w") as f:
            json.dump(self.steps + [self.averages()], f, indent=2)
