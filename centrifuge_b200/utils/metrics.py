"""Training metrics: JSONL + CSV + (optional) TensorBoard, written by rank 0.

Keeps the reference's metric names (train.py:289-320): ``train/loss/train``,
``train/loss/train_all_token``, ``train/timer/<phase>``, ``eval/loss``, ``eval/perplexity``,
plus ``train/tokens_per_s`` (device-timed) and ``train/kept_ratio``.
"""
from __future__ import annotations

import csv
import json
import os
from typing import Dict, Iterable, Optional, Tuple


class MetricsWriter:
    def __init__(self, out_dir: Optional[str], rank: int = 0, tensorboard: bool = True):
        self.enabled = rank == 0 and out_dir is not None
        self.out_dir = out_dir
        self._jsonl = self._csv = self._tb = None
        if not self.enabled:
            return
        os.makedirs(out_dir, exist_ok=True)
        self._jsonl = open(os.path.join(out_dir, "metrics.jsonl"), "a")
        self._csv_f = open(os.path.join(out_dir, "metrics.csv"), "a", newline="")
        self._csv = csv.writer(self._csv_f)
        if tensorboard:
            try:
                from torch.utils.tensorboard import SummaryWriter
                self._tb = SummaryWriter(os.path.join(out_dir, "tensorboard"))
            except Exception:
                self._tb = None

    def write_events(self, events: Iterable[Tuple[str, float, int]]) -> None:
        if not self.enabled:
            return
        for name, value, step in events:
            self._jsonl.write(json.dumps({"name": name, "value": value, "step": step}) + "\n")
            self._csv.writerow([name, value, step])
            if self._tb is not None:
                self._tb.add_scalar(name, value, step)
        self._jsonl.flush()
        self._csv_f.flush()

    def log(self, step: int, values: Dict[str, float]) -> None:
        self.write_events((k, float(v), step) for k, v in values.items())

    def close(self) -> None:
        if not self.enabled:
            return
        self._jsonl.close()
        self._csv_f.close()
        if self._tb is not None:
            self._tb.close()
