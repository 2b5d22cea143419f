"""Synthetic training data of the benchmark workloads.

Token ids are uniform over the vocabulary; the per-token reference loss is LogNormal(mu, sigma)
(mu = 1.0, sigma = 0.5 by default) -- the shape of a real reference-model loss, which is what
the utility-based selection consumes.  The reference's own efficiency benchmark builds synthetic
ids with an all-zero ref_loss (train.py:388-413, data/build_data.py:15-25); ``zero_ref=True``
reproduces that.

Batches are produced on the host in pinned memory, so that a training step includes the
host-to-device copy of its inputs, as real training does.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator, Optional

import torch


@dataclass
class Batch:
    input_ids: torch.Tensor  # [B, S] int64
    ref_loss: torch.Tensor  # [B, S-1] fp32
    attention_mask: Optional[torch.Tensor] = None  # [B, S] int64, None = all ones

    def to(self, device, non_blocking=True) -> "Batch":
        am = None if self.attention_mask is None else self.attention_mask.to(device, non_blocking=non_blocking)
        return Batch(self.input_ids.to(device, non_blocking=non_blocking),
                     self.ref_loss.to(device, non_blocking=non_blocking), am)

    def nbytes(self) -> int:
        n = self.input_ids.numel() * self.input_ids.element_size()
        n += self.ref_loss.numel() * self.ref_loss.element_size()
        if self.attention_mask is not None:
            n += self.attention_mask.numel() * self.attention_mask.element_size()
        return n


class SyntheticTokenData:
    def __init__(self, vocab_size: int, batch_size: int, seq_len: int, seed: int = 4321,
                 mu: float = 1.0, sigma: float = 0.5, zero_ref: bool = False, pin: bool = True,
                 rank: int = 0):
        self.vocab_size, self.B, self.S = vocab_size, batch_size, seq_len
        self.mu, self.sigma, self.zero_ref = mu, sigma, zero_ref
        self.gen = torch.Generator().manual_seed(seed + 1000003 * rank)
        self.pin = pin and torch.cuda.is_available()

    def sample(self) -> Batch:
        ids = torch.randint(0, self.vocab_size, (self.B, self.S), generator=self.gen)
        if self.zero_ref:
            ref = torch.zeros(self.B, self.S - 1)
        else:
            z = torch.randn(self.B, self.S - 1, generator=self.gen)
            ref = torch.exp(self.mu + self.sigma * z)
        if self.pin:
            ids, ref = ids.pin_memory(), ref.pin_memory()
        return Batch(ids, ref)

    def __iter__(self) -> Iterator[Batch]:
        while True:
            yield self.sample()


def create_synthetic_data(num_samples: int, seq_len: int, vocab_size: int, seed: int = 4321):
    """List of ``{"input_ids", "attention_mask", "ref_loss"}`` dicts (reference
    data/build_data.py:15-25 layout) for the dataset/collate path."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(num_samples):
        ids = torch.randint(0, vocab_size, (seq_len,), generator=g).tolist()
        out.append({"input_ids": ids, "attention_mask": [1] * seq_len,
                    "ref_loss": [0.0] * (seq_len - 1)})
    return out
