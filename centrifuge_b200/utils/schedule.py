"""Learning-rate schedule: linear warm-up then cosine decay to ``cos_min_ratio * lr``.

Same shape as the DeepSpeed ``WarmupCosineLR`` the reference configures (train.py:136-145:
``warmup_min_ratio 0``, ``cos_min_ratio 0.1``, warm-up over 5% of the steps).
"""
from __future__ import annotations

import math


class WarmupCosineLR:
    def __init__(self, base_lr: float, total_steps: int, warmup_steps: int,
                 cos_min_ratio: float = 0.1, warmup_min_ratio: float = 0.0):
        self.base_lr = base_lr
        self.total = max(1, total_steps)
        self.warmup = max(0, warmup_steps)
        self.cos_min = cos_min_ratio
        self.warm_min = warmup_min_ratio

    def __call__(self, step: int) -> float:
        if self.warmup > 0 and step < self.warmup:
            r = self.warm_min + (1 - self.warm_min) * step / self.warmup
            return self.base_lr * r
        prog = min(1.0, (step - self.warmup) / max(1, self.total - self.warmup))
        ratio = self.cos_min + (1 - self.cos_min) * 0.5 * (1 + math.cos(math.pi * prog))
        return self.base_lr * ratio


def layer_lr_scales(num_layers: int, decay: float):
    """Per-layer learning-rate multipliers (reference train.py:55-77): ``lm_head`` 1.0,
    ``embed_tokens`` ``1/decay``, layer ``i`` (1-based) ``1 + (1 - i/L) * (1/decay - 1)``."""
    inc = 1.0 / decay
    scales = {"lm_head": 1.0, "norm": 1.0, "embed": inc}
    for i in range(num_layers):
        scales[f"layers.{i}"] = 1.0 + (1 - (i + 1) / num_layers) * (inc - 1)
    return scales
