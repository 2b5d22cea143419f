"""Pipeline parallelism: 1F1B schedule over TP x PP ranks with the filtered backward.

Reference status: PP/1F1B exists only through stock Megatron ``pretrain`` (never with the
filter on the real path) and a forward-only stage demo (megatronlm/
megatron_tinyllama_pp_graph.py:345-420, even split ``layers_per_stage + (stage < rem)``).

Here every stage is a :class:`~centrifuge_b200.models.tp_llama.TPLlamaCore` holding its layer
range (embedding on the first stage, norm + LM head on the last).  Ranks are laid out
``rank = stage * TP + tp_rank``; stage ``s`` rank ``t`` talks to stage ``s+-1`` rank ``t``.

Per micro-batch the last stage computes the per-token loss, the selection mask and the filtered
backward.  The mask is sent back with the gradient, so earlier stages build the same kept-row
layout; backward point-to-point messages carry only the (padded) kept rows ``[C, H]`` of the
sequence shard, forward messages the full shard ``[T/TP, H]``.  Sends are non-blocking
(NCCL / gloo ``isend``), receives are waited in schedule order, which keeps the 1F1B order
deadlock-free.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from ..filter import backward_filter
from ..filter.state import FilterState, state_for_mask
from ..loss import keep_count, token_filter_loss
from .tensor_parallel import KeptLayout


def stage_layers(num_layers: int, pp: int, stage: int) -> range:
    per, rem = divmod(num_layers, pp)
    start = stage * per + min(stage, rem)
    return range(start, start + per + (1 if stage < rem else 0))


@dataclass
class PPGroups:
    tp_group: object
    stage: int
    pp: int
    tp: int
    tp_rank: int
    prev: Optional[int]  # global rank of the same TP rank in the previous stage
    next: Optional[int]


def build_groups(tp: int, pp: int) -> PPGroups:
    """Create the TP groups of every stage (collective over all ranks) and locate neighbours."""
    world, rank = dist.get_world_size(), dist.get_rank()
    assert world == tp * pp, f"world {world} != tp {tp} x pp {pp}"
    mine = None
    for s in range(pp):
        g = dist.new_group(list(range(s * tp, (s + 1) * tp)))
        if rank // tp == s:
            mine = g
    stage, t = rank // tp, rank % tp
    return PPGroups(mine, stage, pp, tp, t, (stage - 1) * tp + t if stage > 0 else None,
                    (stage + 1) * tp + t if stage < pp - 1 else None)


class PipelineTrainer:
    """1F1B training step of one pipeline stage (this process)."""

    def __init__(self, core, optimizer, groups: PPGroups, drop_rate: float = 0.5,
                 strategy: str = "fixed", num_microbatches: int = 8,
                 check_device_errors: bool = True):
        self.core, self.opt, self.g = core, optimizer, groups
        self.drop_rate, self.strategy, self.M = drop_rate, strategy, num_microbatches
        self.first = groups.stage == 0
        self.last = groups.stage == groups.pp - 1
        self.device = core.device
        self._sends: List = []
        # device errors (bounded waits that ran out, bad masks) surface one step late
        self.status = None
        if check_device_errors and torch.device(self.device).type == "cuda":
            from ..utils.device_status import DeviceStatus
            self.status = DeviceStatus(self.device)

    # ------------------------------------------------------------------ p2p
    def _isend(self, t: torch.Tensor, dst: int) -> None:
        self._sends.append((dist.isend(t.contiguous(), dst), t))

    def _recv(self, shape, dtype, src: int) -> torch.Tensor:
        t = torch.empty(shape, dtype=dtype, device=self.device)
        dist.irecv(t, src).wait()
        return t

    def _drain_sends(self) -> None:
        for w, _ in self._sends:
            w.wait()
        self._sends.clear()

    # ------------------------------------------------------------------ stages
    def _forward(self, batch):
        ids, ref = batch
        B, S = ids.shape
        T = B * S
        H = self.core.cfg.hidden_size
        hidden = None
        if not self.first:
            hidden = self._recv((T // self.g.tp, H), self.core.flat.data.dtype, self.g.prev)
        out = self.core(input_ids=ids, hidden=hidden, batch_shape=(B, S))
        if not self.last:
            self._isend(out.hidden.detach(), self.g.next)
            return {"ids": ids, "out": out, "B": B, "S": S}
        mask = torch.ones(B, S, dtype=torch.long, device=self.device)
        if self.drop_rate > 0:
            loss, mask = token_filter_loss(ids, None, mask, ref, self.strategy, self.drop_rate,
                                           True, True, per_token_loss=out.token_loss)
            mask._cf_keep = keep_count(S, self.drop_rate)
            backward_filter(loss, mask)
        else:
            loss = token_filter_loss(ids, None, mask, None, None, None, True,
                                     per_token_loss=out.token_loss)
        return {"ids": ids, "loss": loss, "mask": mask, "B": B, "S": S}

    def _backward(self, st):
        B, S = st["B"], st["S"]
        H = self.core.cfg.hidden_size
        if self.last:
            self.core.pending_input_grad = None
            st["loss"].backward()
            dx = self.core.pending_input_grad
            mask = st["mask"]
        else:
            mask = self._recv((B, S), torch.long, self.g.next)
            filtered = bool(self.drop_rate > 0)
            if filtered and self.strategy == "fixed":
                # every row keeps S - k tokens, known statically: no host read of the mask
                mask._cf_keep = keep_count(S, self.drop_rate)
            state = state_for_mask(mask) if filtered else None
            lay = KeptLayout(state.rows if state is not None else None, B * S,
                             self.core.tp, self.device)
            grad = self._recv((lay.C, H), self.core.flat.data.dtype, self.g.next)
            fn = st["out"].hidden.grad_fn
            sv = fn.saved if fn is not None else None
            dx = self.core._backward_impl(sv, grad, state)
            if fn is not None:
                fn.saved = None
        if not self.first:
            self._isend(mask, self.g.prev)
            self._isend(dx, self.g.prev)
        return st.get("loss")

    # ------------------------------------------------------------------ schedule
    def train_step(self, batches) -> Optional[torch.Tensor]:
        """``batches``: ``M`` pairs ``(input_ids [B, S], ref_loss [B, S-1])`` (same on every
        rank).  Returns the mean loss on the last stage, None elsewhere."""
        M = len(batches)
        warm = min(self.g.pp - self.g.stage - 1, M)
        q = deque()
        losses = []
        fi = 0
        for _ in range(warm):
            q.append(self._forward(batches[fi]))
            fi += 1
        for _ in range(M - warm):
            q.append(self._forward(batches[fi]))
            fi += 1
            l = self._backward(q.popleft())
            if l is not None:
                losses.append(l.detach())
        while q:
            l = self._backward(q.popleft())
            if l is not None:
                losses.append(l.detach())
        self._drain_sends()
        self.core.reduce_replicated_grads()
        self.opt.step(grad_scale=1.0 / M)
        self.opt.zero_grad()
        if self.status is not None:
            self.status.record()
        return torch.stack(losses).mean() if losses else None
