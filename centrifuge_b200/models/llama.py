"""Native Llama for filtered training on B200.

The whole forward and backward of a model (or of one pipeline stage) is ONE autograd node whose
backward runs the sm_100a kernels directly on the kept rows.  The node understands the filter
state that :func:`centrifuge_b200.filter.backward_filter` attaches to it:

* unfiltered: every token row is processed (ordinary dense backward);
* filtered:   only the ``B * S_keep`` kept rows are processed.  Saved activations are read at
  the kept rows (row-index gathers feeding the GEMMs), the lm_head / MLP / projection dgrad
  and wgrad GEMMs run with ``M = B*S_keep`` (dgrad) or ``K = B*S_keep`` (wgrad), and attention
  uses the fused restore-Q backward (kept-key dK/dV, dQ over every key by original position).

This is the B200 equivalent of what the reference reaches by rewriting generic autograd nodes
(grad_filter/token_filter/csrc/node_processing.cpp:65-427 and backward_filters.cpp:420-505):
the same gradients (K/V of dropped positions are constants for the backward; nothing reaches a
dropped position), without per-node saved-tensor surgery or host synchronisation.

Layer math (HF ``LlamaForCausalLM``):
  h = x + o_proj(attn(rope(q), rope(k), v)),  q/k/v = proj(rmsnorm(x))
  y = h + down(silu(gate(rmsnorm(h))) * up(rmsnorm(h)))
Weights are stored fused (``wqkv = [q; k; v]``, ``wgu = [gate; up]``) in one flat bf16 buffer;
:mod:`centrifuge_b200.utils.checkpoint` maps them to and from HF state-dict names.
"""
from __future__ import annotations

import os

import math
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Tuple

import torch

from ..config import LlamaConfig
from ..filter.state import FilterSlot, FilterState
from ..ops import fused
from ..ops import gemm as G
from ..ops.reference import rope_table
from .flat import FlatParams


@dataclass
class CausalLMOutput:
    token_loss: Optional[torch.Tensor] = None  # [B, S-1] fp32 (last stage)
    hidden: Optional[torch.Tensor] = None  # [B*S, H] (non-last pipeline stage)
    logits: Optional[torch.Tensor] = None  # [B, S, V] bf16 view, when kept

    @property
    def loss(self):
        return self.token_loss


def param_specs(cfg: LlamaConfig, layers: range, has_embed: bool, has_head: bool,
                tp: int = 1) -> List[Tuple[str, Tuple[int, ...]]]:
    """Names/shapes of one stage's (tensor-parallel shard of the) parameters, in gradient-
    completion order (head first, embedding last)."""
    H, F, hd = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    nh, nkv = cfg.num_attention_heads // tp, cfg.num_key_value_heads // tp
    V = cfg.vocab_size // tp if tp > 1 else cfg.vocab_size
    specs = []
    if has_head:
        specs.append(("lm_head", (V, H)))
        specs.append(("norm", (H,)))
    for i in reversed(layers):
        p = f"layers.{i}."
        specs += [(p + "wd", (H, F // tp)), (p + "wgu", (2 * (F // tp), H)),
                  (p + "ln2", (H,)), (p + "wo", (H, nh * hd)),
                  (p + "wqkv", ((nh + 2 * nkv) * hd, H)), (p + "ln1", (H,))]
    if has_embed:
        specs.append(("embed", (cfg.vocab_size, H)))
    return specs


class _Saved:
    """Activations of one micro-batch kept for the backward."""

    def __init__(self):
        self.layers: List[Dict[str, torch.Tensor]] = []


class LlamaCore(torch.nn.Module):
    """Layers ``[first, last)`` of a Llama, optionally with embedding and/or LM head."""

    def __init__(self, cfg: LlamaConfig, device="cuda", first: int = 0, last: Optional[int] = None,
                 has_embed: bool = True, has_head: bool = True, seed: int = 0,
                 init: bool = True, keep_logits: bool = False, dtype=torch.bfloat16,
                 pad_to: int = 1, bucket_numel: int = 1 << 26):
        super().__init__()
        assert not cfg.tie_word_embeddings, "tied embeddings are not supported"
        self.cfg = cfg
        self.first = first
        self.last = cfg.num_hidden_layers if last is None else last
        self.layer_ids = range(self.first, self.last)
        self.has_embed, self.has_head = has_embed, has_head
        self.keep_logits = keep_logits
        # CUDA: lm_head + cross entropy fused (no [T, V] logits kept between forward and
        # backward; the kept rows' logits are recomputed).  CFB_FUSED_CE=0 keeps the logits.
        self.fused_ce = os.environ.get("CFB_FUSED_CE", "1") != "0"
        # with data parallelism (pad_to > 1) the layout is cut into reduce-scatter buckets
        self.flat = FlatParams(param_specs(cfg, self.layer_ids, has_embed, has_head), device,
                               dtype=dtype, pad_to=pad_to, bucket_numel=bucket_numel)
        self.device = self.flat.device
        self.nh, self.nkv, self.hd = cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim
        self.scale = 1.0 / math.sqrt(self.hd)
        self._rope = rope_table(cfg.max_position_embeddings, self.hd, cfg.rope_theta,
                                self.device)
        self._pos_cache: Dict[Tuple[int, int], torch.Tensor] = {}
        # Called as hook(lo, hi) when grads of flat[lo:hi] are final for this micro-batch.
        self.grad_ready_hook: Optional[Callable[[int, int], None]] = None
        # Anchor that makes the node's output require grad (the weights are not autograd
        # leaves: their gradients go straight into the flat fp32 buffer).
        self._anchor = torch.zeros((), device=self.device, requires_grad=True)
        if init:
            self.reset_parameters(seed)

    # ------------------------------------------------------------------ parameters
    def reset_parameters(self, seed: int = 0) -> None:
        """HF Llama init: N(0, initializer_range) for matrices, ones for norms."""
        g = torch.Generator(device=self.device).manual_seed(seed)
        std = self.cfg.initializer_range
        for name, p in self.flat.params.items():
            if p.dim() == 1:
                p.fill_(1.0)
            else:
                p.normal_(0.0, std, generator=g)

    def named_flat_parameters(self):
        return self.flat.params.items()

    def _pos(self, B: int, S: int) -> torch.Tensor:
        key = (B, S)
        t = self._pos_cache.get(key)
        if t is None:
            t = torch.arange(S, dtype=torch.int32, device=self.device).repeat(B)
            self._pos_cache[key] = t
        return t

    # ------------------------------------------------------------------ forward
    def forward(self, input_ids: Optional[torch.Tensor] = None,
                hidden: Optional[torch.Tensor] = None, labels: Optional[torch.Tensor] = None,
                batch_shape: Optional[Tuple[int, int]] = None) -> CausalLMOutput:
        """``input_ids [B, S]`` (first stage) or ``hidden [B*S, H]`` (later stages)."""
        if self.has_embed:
            B, S = input_ids.shape
        else:
            B, S = batch_shape
        out = _CfLlamaFn.apply(self._anchor, hidden, input_ids, labels, self, B, S)
        if self.has_head:
            res = CausalLMOutput(token_loss=out)
            if self.keep_logits and getattr(self, "_last_logits", None) is not None:
                res.logits = self._last_logits.view(B, S, -1)
            return res
        return CausalLMOutput(hidden=out)

    def _forward_impl(self, input_ids, hidden_in, labels, B, S) -> Tuple[torch.Tensor, _Saved]:
        p = self.flat.params
        cfg = self.cfg
        H = cfg.hidden_size
        T = B * S
        nh, nkv, hd = self.nh, self.nkv, self.hd
        sv = _Saved()
        sv.B, sv.S = B, S
        pos = self._pos(B, S)
        if self.has_embed:
            ids = input_ids.reshape(-1).contiguous()
            sv.ids = ids
            x = fused.embedding_fwd(p["embed"], ids)
        else:
            x = hidden_in.contiguous()
        for i in self.layer_ids:
            pre = f"layers.{i}."
            L = {"x": x}
            xn, rstd1 = fused.rmsnorm_fwd(x, p[pre + "ln1"], cfg.rms_norm_eps)
            # RoPE of the q and k heads runs in the projection's epilogue
            qkv = G.linear_fwd_rope(xn, p[pre + "wqkv"], pos, self._rope, (nh + nkv) * hd, hd)
            o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd, scale=self.scale)
            x2 = G.linear_fwd(o, p[pre + "wo"], resid=x)
            xn2, rstd2 = fused.rmsnorm_fwd(x2, p[pre + "ln2"], cfg.rms_norm_eps)
            gu, h = G.linear_fwd_swiglu(xn2, p[pre + "wgu"])  # SwiGLU in the epilogue
            x = G.linear_fwd(h, p[pre + "wd"], resid=x2)
            L.update(xn=xn, rstd1=rstd1, qkv=qkv, o=o, lse=lse, x2=x2, xn2=xn2, rstd2=rstd2,
                     gu=gu, h=h)
            sv.layers.append(L)
        if not self.has_head:
            return x, sv
        xf, rstdf = fused.rmsnorm_fwd(x, p["norm"], cfg.rms_norm_eps)
        if labels is None:
            lab = torch.full((B, S), -100, dtype=torch.long, device=x.device)
            lab[:, :-1] = input_ids[:, 1:]
        else:
            lab = labels.to(torch.long).clone()
        lab = lab.reshape(-1).contiguous()
        if self.fused_ce and x.is_cuda and not self.keep_logits:
            # lm_head GEMM with the cross-entropy statistics in its epilogue: the [T, V] logits
            # are never stored; the backward recomputes them for the kept rows only
            logits = None
            loss, lse_ce = G.linear_fwd_ce(xf, p["lm_head"], lab)
        else:
            logits = G.linear_fwd(xf, p["lm_head"])
            loss, lse_ce = fused.ce_fwd(logits, lab)
        sv.head = dict(x=x, xf=xf, rstdf=rstdf, logits=logits, labels=lab, lse=lse_ce)
        self._last_logits = logits if self.keep_logits else None
        token_loss = loss.view(B, S)[:, :-1].contiguous()
        return token_loss, sv

    # ------------------------------------------------------------------ backward
    def _gather(self, t: torch.Tensor, rows: Optional[torch.Tensor]) -> torch.Tensor:
        return t if rows is None else fused.gather_rows(t, rows)

    def _notify(self, *names: str) -> None:
        if self.grad_ready_hook is None:
            return
        lo = min(self.flat.offsets[n] for n in names)
        hi = max(self.flat.range_of(n)[1] for n in names)
        self.grad_ready_hook(lo, hi)

    def _backward_impl(self, sv: _Saved, grad_out: torch.Tensor,
                       state: Optional[FilterState]) -> Optional[torch.Tensor]:
        p, g = self.flat.params, self.flat.grads
        cfg = self.cfg
        B, S = sv.B, sv.S
        nh, nkv, hd = self.nh, self.nkv, self.hd
        if state is not None:
            assert state.B == B and state.S == S, "filter mask does not match the batch"
            rows, Sk = state.rows, state.s_keep
            pos_flat, pos2d = state.pos_flat, state.pos
        else:
            rows, Sk = None, S
            pos_flat, pos2d = self._pos(B, S), None
        Tk = B * Sk
        if self.has_head:
            hd_ = sv.head
            dl = grad_out.float()
            if state is not None and dl.shape[1] == S - 1:
                # the loss nodes above were not rewritten: pick the kept loss positions
                idx = pos2d[:, :-1].long()
                dl = torch.gather(dl, 1, idx)
            dl = torch.cat([dl, torch.zeros(B, 1, device=dl.device, dtype=dl.dtype)], 1)
            dloss = dl.reshape(-1).contiguous()
            xf_k = self._gather(hd_["xf"], rows)
            if hd_["logits"] is None:
                # recompute the kept rows' logits inside the GEMM; its epilogue writes dlogits
                lab_k, lse_k = hd_["labels"], hd_["lse"]
                if rows is not None:
                    lab_k, lse_k = lab_k[rows.long()], lse_k[rows.long()]
                dlogits = G.linear_ce_grad(xf_k, p["lm_head"], lab_k, lse_k, dloss)
            else:
                dlogits = fused.ce_bwd(hd_["logits"], hd_["labels"], hd_["lse"], dloss, rows)
            G.linear_wgrad(dlogits, xf_k, g["lm_head"])
            dxf = G.linear_dgrad(dlogits, p["lm_head"])
            del dlogits, xf_k
            dx = fused.rmsnorm_bwd(dxf, hd_["x"], hd_["rstdf"], p["norm"], g["norm"], x_rows=rows)
            self._notify("lm_head", "norm")
        else:
            dx = grad_out.contiguous()
            if dx.shape[0] != Tk:
                dx = self._gather(dx, rows)
        for li, i in reversed(list(enumerate(self.layer_ids))):
            L = sv.layers[li]
            pre = f"layers.{i}."
            # ---- MLP
            dh = G.linear_dgrad(dx, p[pre + "wd"])
            # a separate pass: the SwiGLU backward in the dgrad epilogue (linear_dgrad_swiglu)
            # measured slower at these shapes (its gathered gate/up reads stall the epilogue).
            # The pass also recomputes h of the kept rows from the gate / up it reads anyway,
            # which replaces a gather of h for the down projection's weight gradient.
            if rows is None:
                h_k = L["h"]
                dgu = fused.swiglu_bwd(dh, L["gu"], None)
            else:
                h_k = torch.empty_like(dh)
                dgu = fused.swiglu_bwd(dh, L["gu"], rows, h_out=h_k)
            del dh
            G.linear_wgrad(dx, h_k, g[pre + "wd"])
            del h_k
            xn2_k = self._gather(L["xn2"], rows)
            G.linear_wgrad(dgu, xn2_k, g[pre + "wgu"])
            dxn2 = G.linear_dgrad(dgu, p[pre + "wgu"])
            del dgu, xn2_k
            dx2 = fused.rmsnorm_bwd(dxn2, L["x2"], L["rstd2"], p[pre + "ln2"], g[pre + "ln2"],
                                    x_rows=rows, dres=dx)
            del dxn2, dx
            # ---- attention
            o_k = self._gather(L["o"], rows)
            G.linear_wgrad(dx2, o_k, g[pre + "wo"])
            do = G.linear_dgrad(dx2, p[pre + "wo"])
            qkv_k = self._gather(L["qkv"], rows)
            lse_k = self._gather(L["lse"], rows)
            dqkv = fused.attn_bwd(qkv_k, L["qkv"], o_k, do, lse_k,
                                  pos2d if pos2d is not None else pos_flat.view(B, S),
                                  B, S, Sk, nh, nkv, hd, scale=self.scale,
                                  rope_table=self._rope)  # RoPE backward in the epilogue
            del qkv_k, lse_k, o_k, do
            xn_k = self._gather(L["xn"], rows)
            G.linear_wgrad(dqkv, xn_k, g[pre + "wqkv"])
            dxn = G.linear_dgrad(dqkv, p[pre + "wqkv"])
            del dqkv, xn_k
            dx = fused.rmsnorm_bwd(dxn, L["x"], L["rstd1"], p[pre + "ln1"], g[pre + "ln1"],
                                   x_rows=rows, dres=dx2)
            del dxn, dx2
            sv.layers[li] = None
            self._notify(pre + "wd", pre + "wgu", pre + "ln2", pre + "wo", pre + "wqkv",
                         pre + "ln1")
        if self.has_embed:
            fused.embedding_bwd(dx, sv.ids, g["embed"], id_rows=rows)
            self._notify("embed")
            return None
        return dx


class _CfLlamaFn(torch.autograd.Function):
    """Autograd node of a native Llama stage.  Its backward node is named
    ``_CfLlamaFnBackward``; the graph rewriter recognises the ``_Cf`` prefix and calls
    :meth:`cf_attach` with the keep mask."""

    @staticmethod
    def forward(ctx, anchor, hidden, input_ids, labels, model: LlamaCore, B: int, S: int):
        out, sv = model._forward_impl(input_ids, hidden, labels, B, S)
        ctx.model = model
        ctx.saved = sv
        ctx.slot = FilterSlot()
        ctx.hidden_in = not model.has_embed
        return out

    @staticmethod
    def backward(ctx, grad_out):
        sv = ctx.saved
        ctx.saved = None
        if sv is None:
            raise RuntimeError("native Llama backward ran twice (retain_graph is not supported)")
        dx = ctx.model._backward_impl(sv, grad_out, ctx.slot.state)
        return None, (dx if ctx.hidden_in else None), None, None, None, None, None

    @staticmethod
    def cf_attach(ctx, mask: torch.Tensor) -> None:
        ctx.slot.attach(mask)


class NativeLlamaForCausalLM(LlamaCore):
    """Full model on one device: ``model(input_ids).token_loss`` is ``[B, S-1]``."""

    def __init__(self, cfg: LlamaConfig, device="cuda", seed: int = 0, **kw):
        super().__init__(cfg, device=device, seed=seed, **kw)
