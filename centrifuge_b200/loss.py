"""Per-token causal-LM loss, utility-based token selection and the masked loss average.

Behavioural contract (reference model/utils.py):

* ``causal_modeling_loss`` -- per-token CE of shifted logits, shape ``[B, S-1]``
  (model/utils.py:385-396).
* ``token_dropping_mask`` -- zeroes, in place in the attention mask, the ``k`` loss positions
  with the smallest score for each row.  ``k`` comes from ``align_drop_rate``, which rounds the
  number of dropped tokens up to a multiple of 8 (model/utils.py:398-424).  Strategies:
  ``fixed``, ``positive``, ``self``, ``less_ref``, ``peaking`` (model/utils.py:425-529);
  ``dynamic`` is not implemented in the reference either.
* ``loss_average`` -- per-sample masked mean then batch mean (model/utils.py:295-309).
* ``token_filter_loss`` -- the composition used by the trainers (model/utils.py:311-344).

Mask index convention: position ``i`` of the ``[B, S]`` mask gates the loss of position ``i``
(which predicts token ``i+1``) under left padding; the last position is never dropped.

On CUDA tensors the ``fixed``/``self``/``less_ref`` selection runs as one sm_100a kernel per
batch (a per-row bitonic select, no host synchronisation); on CPU it runs ``torch.topk``.
"""
from __future__ import annotations

import os
from typing import List, Optional, Sequence, Union

import torch

__all__ = [
    "causal_modeling_loss", "loss_average", "is_left_padding", "apply_mask_to_loss",
    "align_drop_rate", "token_dropping_mask", "token_filter_loss", "num_dropped",
    "keep_count", "STRATEGIES",
]

STRATEGIES = ("fixed", "positive", "dynamic", "self", "less_ref", "peaking")


def is_left_padding(attention_mask: torch.Tensor) -> bool:
    """True when padding sits on the left (model/utils.py:260-267)."""
    with torch.no_grad():
        left = attention_mask[:, 0].sum().item()
        right = attention_mask[:, -1].sum().item()
        return left <= right


def causal_modeling_loss(inputs: torch.Tensor, logits: torch.Tensor, attention_mask=None,
                         is_left_padding: Optional[bool] = None, average: bool = False,
                         by_sample: bool = False) -> torch.Tensor:
    """Per-token cross entropy of ``logits[:, :-1]`` against ``inputs[:, 1:]``."""
    labels = inputs[..., 1:].contiguous()
    shifted = logits[..., :-1, :].contiguous()
    loss = torch.nn.functional.cross_entropy(
        shifted.view(-1, shifted.size(-1)).float(), labels.view(-1), reduction="none")
    loss = loss.view(labels.size(0), labels.size(1))
    if not average:
        return loss
    return loss_average(loss, attention_mask, by_sample=by_sample,
                        is_left_padding=is_left_padding)


def apply_mask_to_loss(loss: torch.Tensor, attention_mask: Optional[torch.Tensor]):
    """Multiply the per-token loss by the (left-padded) mask (model/utils.py:288-293)."""
    if attention_mask is None:
        return loss
    if is_left_padding(attention_mask):
        return loss * attention_mask[..., 1:]
    return loss * attention_mask[..., 1:]


def loss_average(loss: torch.Tensor, attention_mask: Optional[torch.Tensor], by_sample=False,
                 is_left_padding: Optional[bool] = None) -> torch.Tensor:
    """Masked per-sample mean, then the batch mean (model/utils.py:295-309)."""
    if attention_mask is not None:
        left = is_left_padding if is_left_padding is not None else globals()["is_left_padding"](
            attention_mask)
        loss_mask = attention_mask[..., :-1] if left else attention_mask[..., 1:]
        loss = torch.multiply(loss, loss_mask)
        loss = loss.sum(-1) / loss_mask.sum(-1)
    else:
        loss = loss.mean(-1)
    return loss if by_sample else loss.mean()


def align_drop_rate(drop_rate: float, seq_len: int, align_div: int = 8) -> float:
    """Round the number of dropped loss tokens up to a multiple of ``align_div``.

    Same float arithmetic as model/utils.py:400-407 so that ``int(rate * seq_len)`` yields the
    aligned count.
    """
    filter_len = int(seq_len * drop_rate)
    if filter_len % align_div != 0:
        filter_len = filter_len + (align_div - (filter_len % align_div))
        return (filter_len / seq_len) + (0.5 / seq_len)
    return drop_rate


def num_dropped(seq_len: int, drop_rate: float, loss_tokens: Optional[int] = None) -> int:
    """Number of positions a full row of length ``seq_len`` drops (``k``)."""
    n_loss = seq_len - 1
    rate = align_drop_rate(drop_rate, n_loss)
    tokens = n_loss if loss_tokens is None else loss_tokens
    return int(rate * tokens)


def keep_count(seq_len: int, drop_rate: float) -> int:
    """``S_keep = S - k`` for an unpadded row (static: no host sync is needed)."""
    return seq_len - num_dropped(seq_len, drop_rate)


def _row_ranges(attention_mask: torch.Tensor, left_padding: bool):
    """Per-row ``(loss_token_size, start, end)`` as in model/utils.py:415-417."""
    S = attention_mask.shape[1]
    sizes = (attention_mask.sum(1) - 1).tolist()
    out = []
    for n in sizes:
        n = int(n)
        start = int(S - n - 1) if left_padding else 1
        end = (S - 1) if left_padding else int(n + 1)
        out.append((n, start, end))
    return out


def _drop_smallest(score: torch.Tensor, attention_mask: torch.Tensor, rate: float,
                   left_padding: bool) -> torch.Tensor:
    """Zero the ``int(rate * n_i)`` smallest scores of each row inside its loss range."""
    B, S = attention_mask.shape
    full = bool((attention_mask.sum(1) == S).all().item()) if B > 0 else True
    if full:
        n = S - 1
        k = int(rate * n)
        start, end = (0, S - 1) if left_padding else (1, S)
        # the score has S-1 columns: right padding's range [1, S) is [1, S-1) in effect, as
        # the reference's slice loss_diff[i][1:S] truncates it (model/utils.py:418)
        end = min(end, int(score.shape[1]))
        if k <= 0:
            return attention_mask
        if attention_mask.is_cuda and k < end - start:
            from .ops import select as _select
            _select.drop_smallest_(score, attention_mask, k, start, end)
            return attention_mask
        _, idx = torch.topk(score[:, start:end], k, dim=1, largest=False)
        attention_mask.scatter_(1, idx + start, 0)
        return attention_mask
    for i, (n, start, end) in enumerate(_row_ranges(attention_mask, left_padding)):
        k = int(rate * n)
        if k <= 0:
            continue
        _, idx = torch.topk(score[i][start:end], k, largest=False)
        attention_mask[i].scatter_(0, idx + start, 0)
    return attention_mask


def _peaking(loss_diff: torch.Tensor, attention_mask: torch.Tensor, drop_rate: float,
             left_padding: bool) -> torch.Tensor:
    """Cluster-anchored selection (model/utils.py:471-527)."""
    for i, (n, start, end) in enumerate(_row_ranges(attention_mask, left_padding)):
        d = loss_diff[i][start:end]
        srt = d.sort(descending=False)[0]
        t40 = srt[int(drop_rate * n)]
        t60 = srt[int(0.6 * n)]
        anchor = d < t40
        cluster = (d < t60).int()
        padded = torch.cat([torch.zeros(1, dtype=cluster.dtype, device=cluster.device), cluster])
        diff = padded[1:] - padded[:-1]
        starts = (diff == 1).nonzero(as_tuple=False).squeeze(-1)
        ends = (diff == -1).nonzero(as_tuple=False).squeeze(-1)
        if len(starts) > len(ends):
            ends = torch.cat([ends, torch.tensor([len(d)], device=ends.device, dtype=torch.long)])
        lengths = ends - starts
        long_enough = lengths >= 3
        sel = torch.zeros_like(cluster, dtype=torch.bool)
        for s, e in zip(starts[long_enough].tolist(), ends[long_enough].tolist()):
            if bool(anchor[s:e].any()):
                sel[s:e] = True
        idx = sel.nonzero(as_tuple=False).squeeze(-1)
        if int(long_enough.sum()) == 0:
            idx = anchor.nonzero(as_tuple=False).squeeze(-1)
        attention_mask[i].scatter_(0, idx + start, 0)
    return attention_mask


def token_dropping_mask(loss: torch.Tensor, ref_loss: Optional[torch.Tensor],
                        attention_mask: torch.Tensor, strategy: str = "fixed",
                        drop_rate: Optional[float] = None,
                        left_padding: Optional[bool] = None,
                        drop_rate_log: Optional[str] = None) -> torch.Tensor:
    """Drop tokens from ``attention_mask`` in place and return it.

    ``loss`` and ``ref_loss`` are ``[B, S-1]``; ``attention_mask`` is ``[B, S]``.
    """
    if strategy not in STRATEGIES:
        raise NotImplementedError(f"Strategy {strategy} is not supported.")
    if strategy == "dynamic":
        raise NotImplementedError(f"Strategy {strategy} is not implemented.")
    left = left_padding if left_padding is not None else is_left_padding(attention_mask)
    seq_len = loss.shape[1]
    with torch.no_grad():
        if strategy == "fixed":
            rate = align_drop_rate(drop_rate, seq_len)
            return _drop_smallest(loss - ref_loss, attention_mask, rate, left)
        if strategy == "positive":
            diff = loss - ref_loss
            negative_rate = float(((diff < 0).sum(1).min() / diff.shape[1]).item())
            rate = max(0.2, min(negative_rate, drop_rate))
            rate = align_drop_rate(rate, seq_len)
            if drop_rate_log is not None:
                os.makedirs(os.path.dirname(drop_rate_log) or ".", exist_ok=True)
                with open(drop_rate_log, "a") as f:
                    f.write(f"drop_rate: {rate}\n")
            return _drop_smallest(diff, attention_mask, rate, left)
        if strategy == "self":
            return _drop_smallest(loss.clone(), attention_mask, drop_rate, left)
        if strategy == "less_ref":
            return _drop_smallest(-1.0 * ref_loss, attention_mask, drop_rate, left)
        # peaking
        return _peaking(loss - ref_loss, attention_mask, drop_rate, left)


def _pad_ref_loss(ref_loss, loss: torch.Tensor) -> torch.Tensor:
    """Left-pad each row of ``ref_loss`` with zeros to the loss length (model/utils.py:321-322)."""
    if isinstance(ref_loss, torch.Tensor):
        r = ref_loss.to(device=loss.device, dtype=loss.dtype)
        if r.shape[1] < loss.shape[1]:
            r = torch.nn.functional.pad(r, (loss.shape[1] - r.shape[1], 0))
        return r
    rows = []
    n = loss.shape[1]
    for r in ref_loss:
        r = list(r)
        rows.append([0.0] * (n - len(r)) + r)
    return torch.tensor(rows, dtype=loss.dtype, device=loss.device)


def token_filter_loss(inputs: torch.Tensor, logits, attention_mask: Optional[torch.Tensor] = None,
                      ref_loss: Union[None, torch.Tensor, Sequence[Sequence[float]]] = None,
                      dropping_strategy: Optional[str] = None, drop_rate: Optional[float] = None,
                      is_left_padding: Optional[bool] = None, return_mask: bool = False,
                      batch_timer=None, per_token_loss: Optional[torch.Tensor] = None):
    """Filtered training loss; optionally returns the selection mask (model/utils.py:311-344).

    ``logits`` may be ``None`` when ``per_token_loss`` (``[B, S-1]``) is given; the native
    models compute it with a fused lm_head + cross-entropy and never materialise the logits
    for the selection step.
    """
    if batch_timer is not None:
        batch_timer.record_nvtx("causal_modeling_loss")
    if per_token_loss is not None:
        loss = per_token_loss
    else:
        loss = causal_modeling_loss(inputs, logits, attention_mask=None, average=False)
    if batch_timer is not None:
        batch_timer.record("causal_modeling_loss")
    if attention_mask is None:
        attention_mask = torch.ones(inputs.shape[0], inputs.shape[1], dtype=torch.long,
                                    device=inputs.device)
    left = is_left_padding if is_left_padding is not None else globals()["is_left_padding"](
        attention_mask)
    if ref_loss is not None:
        if batch_timer is not None:
            batch_timer.record_nvtx("token_dropping_mask")
        ref = _pad_ref_loss(ref_loss, loss.detach())
        if isinstance(ref_loss, list):
            for i in range(len(ref_loss)):
                ref_loss[i] = ref[i].tolist()
        mask = token_dropping_mask(loss.detach(), ref, attention_mask,
                                   strategy=dropping_strategy, drop_rate=drop_rate,
                                   left_padding=left)
        if batch_timer is not None:
            batch_timer.record("token_dropping_mask")
        out = loss_average(loss, mask, by_sample=False, is_left_padding=left)
        return (out, mask) if return_mask else out
    out = loss_average(loss, attention_mask, by_sample=False, is_left_padding=left)
    return (out, attention_mask) if return_mask else out
