"""Device-side token selection: per-row k-smallest drop and kept-index construction.

``drop_smallest_`` zeroes, for every row, the mask at the ``k`` smallest scores inside
``[start, end)`` (model/utils.py:409-424 does this with a per-row ``torch.topk`` loop and host
synchronisations).  ``keep_index`` turns the mask into kept positions and flattened kept-row ids
without a host round trip; the kept count per row is known statically (``S - k``).
"""
from __future__ import annotations

import torch

from ._ext import kernels, status_block


def drop_smallest_(score: torch.Tensor, mask: torch.Tensor, k: int, start: int, end: int):
    score = score.float().contiguous()
    if not score.is_cuda:
        _, idx = torch.topk(score[:, start:end], k, dim=1, largest=False)
        mask.scatter_(1, idx + start, 0)
        return mask
    kernels().drop_smallest(score, mask, start, end, k)
    return mask


def keep_index(mask: torch.Tensor, s_keep: int):
    """``(pos [B, S_keep] int32, flat_rows [B*S_keep] int32, status)``.

    On the GPU ``status`` is the kernels' per-device status block; its word 0 becomes
    ``kErrKeepCount`` (64) when a row does not keep exactly ``s_keep`` tokens (the training loop
    reads it one step late).  On the CPU a wrong count raises at once.
    """
    B, S = mask.shape
    if not mask.is_cuda:
        keep = mask != 0
        counts = keep.sum(1)
        if not bool((counts == s_keep).all()):
            raise ValueError(f"every row must keep {s_keep} tokens, got {counts.tolist()}")
        pos = keep.nonzero()[:, 1].view(B, s_keep).to(torch.int32)
        flat = (pos + (torch.arange(B, dtype=torch.int32) * S).view(B, 1)).reshape(-1)
        return pos, flat, torch.zeros(1, dtype=torch.int32)
    m = mask if mask.dtype == torch.long else mask.long()
    m = m.contiguous()
    pos = torch.empty(B, s_keep, dtype=torch.int32, device=mask.device)
    flat = torch.empty(B * s_keep, dtype=torch.int32, device=mask.device)
    err = status_block(mask.device)
    kernels().keep_index(m, s_keep, pos, flat, err)
    return pos, flat, err
