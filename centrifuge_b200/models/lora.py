"""LoRA adapters for HuggingFace models (the reference uses PEFT: r=64, alpha=128,
dropout 0.1 on q/k/v/o, train.py:88-95).  PEFT is not a dependency here; this wraps the target
``nn.Linear`` modules with a frozen base and trainable low-rank ``A``/``B``, which the graph
rewriter filters like any other backward node (``MmBackward0`` / ``AddmmBackward0``)."""
from __future__ import annotations

import math
from typing import Iterable

import torch
from torch import nn


class LoRALinear(nn.Module):
    def __init__(self, base: nn.Linear, r: int = 64, alpha: int = 128, dropout: float = 0.1):
        super().__init__()
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        self.r, self.scaling = r, alpha / r
        self.lora_A = nn.Parameter(torch.empty(r, base.in_features, dtype=base.weight.dtype,
                                               device=base.weight.device))
        self.lora_B = nn.Parameter(torch.zeros(base.out_features, r, dtype=base.weight.dtype,
                                               device=base.weight.device))
        nn.init.kaiming_uniform_(self.lora_A, a=math.sqrt(5))
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()

    def forward(self, x):
        return self.base(x) + (self.dropout(x) @ self.lora_A.t() @ self.lora_B.t()) * self.scaling


def apply_lora(model: nn.Module, r: int = 64, alpha: int = 128, dropout: float = 0.1,
               targets: Iterable[str] = ("q_proj", "k_proj", "v_proj", "o_proj")) -> nn.Module:
    """Freeze ``model`` and replace each target linear with a :class:`LoRALinear`."""
    targets = set(targets)
    for p in model.parameters():
        p.requires_grad_(False)
    for name, mod in list(model.named_modules()):
        for child_name, child in list(mod.named_children()):
            if child_name in targets and isinstance(child, nn.Linear):
                setattr(mod, child_name, LoRALinear(child, r, alpha, dropout))
    return model
