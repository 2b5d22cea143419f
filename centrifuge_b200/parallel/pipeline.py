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
(NCCL / gloo ``isend``); receives are posted at their use.  ``prefetch`` posts the receives of
a known shape (a forward's input, a backward's mask) one schedule slot ahead instead; measured
slower on B200 (the waiting receive kernels hold SMs), so it is off by default.
"""
from __future__ import annotations

import os
from collections import deque
from dataclasses import dataclass
from typing import List, Optional

import torch
import torch.distributed as dist

from ..filter import backward_filter
from ..filter.state import FilterState, state_for_mask
from ..loss import keep_count, token_filter_loss
from .tensor_parallel import KeptLayout


def stage_layers(num_layers: int, pp: int, stage: int, head_cost: float = 0.0,
                 embed_cost: float = 0.0) -> range:
    """Layer range of pipeline stage ``stage``.

    Without costs: the even split of the reference's stage demo (``per + (stage < rem)``
    layers).  With ``head_cost`` / ``embed_cost`` (the LM head on the last stage and the
    embedding on the first, in units of one decoder layer): contiguous ranges that minimise the
    largest stage cost, every stage keeping at least one layer, so that the stage with the head
    does not set the pipeline's pace alone."""
    if head_cost <= 0.0 and embed_cost <= 0.0:
        per, rem = divmod(num_layers, pp)
        start = stage * per + min(stage, rem)
        return range(start, start + per + (1 if stage < rem else 0))
    assert num_layers >= pp, "every stage needs a layer"
    INF = float("inf")

    def cost(s, a, b):
        return (b - a) + (embed_cost if s == 0 else 0.0) + (head_cost if s == pp - 1 else 0.0)

    # best[s][i]: smallest possible max stage cost when stages 0..s-1 cover layers [0, i)
    best = [[INF] * (num_layers + 1) for _ in range(pp + 1)]
    cut = [[0] * (num_layers + 1) for _ in range(pp + 1)]
    best[0][0] = 0.0
    for s_ in range(1, pp + 1):
        for i in range(s_, num_layers - (pp - s_) + 1):
            for j in range(s_ - 1, i):
                v = max(best[s_ - 1][j], cost(s_ - 1, j, i))
                if v < best[s_][i] - 1e-12:
                    best[s_][i], cut[s_][i] = v, j
    bounds = [num_layers]
    for s_ in range(pp, 0, -1):
        bounds.append(cut[s_][bounds[-1]])
    bounds = bounds[::-1]  # [0, b1, ..., num_layers]
    return range(bounds[stage], bounds[stage + 1])


def head_cost_layers(cfg, seq_len: int) -> float:
    """FLOPs of the LM head (and its loss) per token in units of one decoder layer's FLOPs
    (projections plus causal attention at ``seq_len``)."""
    H, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    hd = getattr(cfg, "head_dim", None) or H // cfg.num_attention_heads
    q, kv = cfg.num_attention_heads * hd, cfg.num_key_value_heads * hd
    layer = H * (q + 2 * kv) + q * H + 3 * H * F + q * seq_len  # causal attention ~ 2 S q / 2
    return V * H / layer


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
        self._pending = {}  # posted receives: (kind, micro-batch) -> (work, tensor)
        # timing=True: CUDA events around every forward / backward compute of this stage
        # (after its receive, before its send), read by busy_ms() to measure the bubble
        self.timing = False
        self._events: List = []
        # prefetch=True (CFB_PP_PREFETCH=1): post the receives of known shape one slot ahead.
        # Off by default: an early receive holds its NCCL kernel on an SM while it waits, which
        # stalls the stage's compute (TP2 x PP2, 16 Llama-3-8B layers, 8 micro-batches: 603 vs
        # 376 ms / step with fused TP collectives, 425 vs 373 ms with NCCL ones).
        self.prefetch = os.environ.get("CFB_PP_PREFETCH", "0") == "1"
        # device errors (bounded waits that ran out, bad masks) surface one step late
        self.status = None
        if check_device_errors and torch.device(self.device).type == "cuda":
            from ..utils.device_status import DeviceStatus
            self.status = DeviceStatus(self.device)

    # ------------------------------------------------------------------ p2p
    # Receives whose shape is known in advance are posted one schedule slot ahead, so the
    # transfer runs under the compute of the slot before: a forward's input activations are
    # posted when the previous forward starts (the previous stage sends them before it needs
    # anything of this micro-batch's backward), a backward's mask right after the send of the
    # forward output that precedes that backward.  Per neighbour the posting order equals the
    # neighbour's send order, so in-order p2p streams (NCCL) cannot deadlock.
    def _isend(self, t: torch.Tensor, dst: int) -> None:
        self._sends.append((dist.isend(t.contiguous(), dst), t))

    def _post(self, key, shape, dtype, src: int) -> None:
        if key not in self._pending:
            t = torch.empty(shape, dtype=dtype, device=self.device)
            self._pending[key] = (dist.irecv(t, src), t)

    def _take(self, key, shape, dtype, src: int) -> torch.Tensor:
        self._post(key, shape, dtype, src)
        w, t = self._pending.pop(key)
        w.wait()
        return t

    def _fwd_shape(self, batch):
        B, S = batch[0].shape
        return (B * S // self.g.tp, self.core.cfg.hidden_size)

    def _mark(self, start=None):
        """Record a CUDA event (``timing`` only); with ``start``, close the interval."""
        if not self.timing or torch.device(self.device).type != "cuda":
            return None
        ev = torch.cuda.Event(enable_timing=True)
        ev.record()
        if start is not None:
            self._events.append((start, ev))
        return ev

    def busy_ms(self) -> float:
        """Device time spent in this stage's forward / backward compute since the last call
        (synchronises); the rest of a step is the pipeline bubble and communication waits."""
        torch.cuda.synchronize(self.device)
        t = sum(a.elapsed_time(b) for a, b in self._events)
        self._events.clear()
        return t

    def _drain_sends(self) -> None:
        for w, _ in self._sends:
            w.wait()
        self._sends.clear()

    # ------------------------------------------------------------------ stages
    def _forward(self, i: int, batches, prefetch_bwd: int = -1):
        ids, ref = batches[i]
        B, S = ids.shape
        dt = self.core.flat.data.dtype
        hidden = None
        if not self.first:
            hidden = self._take(("f", i), self._fwd_shape(batches[i]), dt, self.g.prev)
            if self.prefetch and i + 1 < len(batches):
                self._post(("f", i + 1), self._fwd_shape(batches[i + 1]), dt, self.g.prev)
        t0 = self._mark()
        out = self.core(input_ids=ids, hidden=hidden, batch_shape=(B, S))
        if not self.last:
            self._mark(t0)
            self._isend(out.hidden.detach(), self.g.next)
            if self.prefetch and prefetch_bwd >= 0:
                pb, ps = batches[prefetch_bwd][0].shape
                self._post(("m", prefetch_bwd), (pb, ps), torch.long, self.g.next)
            return {"i": i, "ids": ids, "out": out, "B": B, "S": S}
        mask = torch.ones(B, S, dtype=torch.long, device=self.device)
        if self.drop_rate > 0:
            loss, mask = token_filter_loss(ids, None, mask, ref, self.strategy, self.drop_rate,
                                           True, True, per_token_loss=out.token_loss)
            mask._cf_keep = keep_count(S, self.drop_rate)
            backward_filter(loss, mask)
        else:
            loss = token_filter_loss(ids, None, mask, None, None, None, True,
                                     per_token_loss=out.token_loss)
        self._mark(t0)
        return {"i": i, "ids": ids, "loss": loss, "mask": mask, "B": B, "S": S}

    def _backward(self, st):
        B, S = st["B"], st["S"]
        H = self.core.cfg.hidden_size
        if self.last:
            t0 = self._mark()
            self.core.pending_input_grad = None
            st["loss"].backward()
            dx = self.core.pending_input_grad
            mask = st["mask"]
            self._mark(t0)
        else:
            mask = self._take(("m", st["i"]), (B, S), torch.long, self.g.next)
            filtered = bool(self.drop_rate > 0)
            if filtered and self.strategy == "fixed":
                # every row keeps S - k tokens, known statically: no host read of the mask
                mask._cf_keep = keep_count(S, self.drop_rate)
            state = state_for_mask(mask) if filtered else None
            lay = KeptLayout(state.rows if state is not None else None, B * S,
                             self.core.tp, self.device)
            grad = self._take(("g", st["i"]), (lay.C, H), self.core.flat.data.dtype, self.g.next)
            fn = st["out"].hidden.grad_fn
            sv = fn.saved if fn is not None else None
            t0 = self._mark()
            dx = self.core._backward_impl(sv, grad, state)
            self._mark(t0)
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
        self._pending = {}
        q = deque()
        losses = []
        for fi in range(warm):
            q.append(self._forward(fi, batches))
        for k in range(M - warm):
            # the backward that follows this forward is micro-batch k: post its mask now
            q.append(self._forward(warm + k, batches, prefetch_bwd=k))
            l = self._backward(q.popleft())
            if l is not None:
                losses.append(l.detach())
        while q:
            l = self._backward(q.popleft())
            if l is not None:
                losses.append(l.detach())
        assert not self._pending, f"unconsumed pipeline receives: {sorted(self._pending)}"
        self._drain_sends()
        self.core.reduce_replicated_grads()
        self.opt.step(grad_scale=1.0 / M)
        self.opt.zero_grad()
        if self.status is not None:
            self.status.record()
        return torch.stack(losses).mean() if losses else None
