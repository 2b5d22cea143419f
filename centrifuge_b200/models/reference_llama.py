"""Plain-PyTorch Llama: the filtered-gradient oracle.

HF ``LlamaForCausalLM`` math and state-dict names, written with ordinary autograd ops.  With
``keep_mask`` given, K and V of dropped positions are detached after RoPE (before attention).
Autograd of the mask-weighted loss through this model is, by construction, the gradient the
filtered backward must produce: no gradient reaches a dropped position, and the dQ of a kept
query still sums over every key (the reference's RESTORE_Q semantics,
grad_filter/token_filter/csrc/backward_filters.cpp:420-505).
"""
from __future__ import annotations

import math
from typing import Dict, Optional

import torch
import torch.nn.functional as F
from torch import nn

from ..config import LlamaConfig


class RMSNorm(nn.Module):
    def __init__(self, h: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(h))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        xf = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * xf.to(x.dtype)


def rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


class Attention(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        H, hd = cfg.hidden_size, cfg.head_dim
        self.q_proj = nn.Linear(H, cfg.num_attention_heads * hd, bias=False)
        self.k_proj = nn.Linear(H, cfg.num_key_value_heads * hd, bias=False)
        self.v_proj = nn.Linear(H, cfg.num_key_value_heads * hd, bias=False)
        self.o_proj = nn.Linear(cfg.num_attention_heads * hd, H, bias=False)

    def forward(self, x, cos, sin, keep_mask: Optional[torch.Tensor]):
        B, S, _ = x.shape
        nh, nkv, hd = self.cfg.num_attention_heads, self.cfg.num_key_value_heads, self.cfg.head_dim
        q = self.q_proj(x).view(B, S, nh, hd).transpose(1, 2)
        k = self.k_proj(x).view(B, S, nkv, hd).transpose(1, 2)
        v = self.v_proj(x).view(B, S, nkv, hd).transpose(1, 2)
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
        if keep_mask is not None:
            km = keep_mask.bool().view(B, 1, S, 1)
            k = torch.where(km, k, k.detach())
            v = torch.where(km, v, v.detach())
        rep = nh // nkv
        k = k.repeat_interleave(rep, dim=1)
        v = v.repeat_interleave(rep, dim=1)
        s = (q @ k.transpose(-1, -2)) / math.sqrt(hd)
        causal = torch.ones(S, S, dtype=torch.bool, device=x.device).triu(1)
        s = s.masked_fill(causal, float("-inf"))
        p = torch.softmax(s.float(), dim=-1).to(q.dtype)
        o = (p @ v).transpose(1, 2).reshape(B, S, nh * hd)
        return self.o_proj(o)


class MLP(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.gate_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.up_proj = nn.Linear(cfg.hidden_size, cfg.intermediate_size, bias=False)
        self.down_proj = nn.Linear(cfg.intermediate_size, cfg.hidden_size, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class Layer(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.self_attn = Attention(cfg)
        self.mlp = MLP(cfg)
        self.input_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)
        self.post_attention_layernorm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)

    def forward(self, x, cos, sin, keep_mask):
        x = x + self.self_attn(self.input_layernorm(x), cos, sin, keep_mask)
        return x + self.mlp(self.post_attention_layernorm(x))


class _Inner(nn.Module):
    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size)
        self.layers = nn.ModuleList(Layer(cfg) for _ in range(cfg.num_hidden_layers))
        self.norm = RMSNorm(cfg.hidden_size, cfg.rms_norm_eps)


class ReferenceLlama(nn.Module):
    """``forward(ids, keep_mask=None) -> logits [B, S, V]``."""

    def __init__(self, cfg: LlamaConfig):
        super().__init__()
        self.cfg = cfg
        self.model = _Inner(cfg)
        self.lm_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False)

    def rope(self, S: int, device, dtype):
        hd = self.cfg.head_dim
        inv = 1.0 / (self.cfg.rope_theta ** (torch.arange(0, hd, 2, dtype=torch.int64).float() / hd))
        t = torch.arange(S, dtype=torch.float32)
        f = torch.outer(t, inv)
        emb = torch.cat([f, f], dim=-1)
        return emb.cos().to(device, dtype), emb.sin().to(device, dtype)

    def forward(self, input_ids, keep_mask: Optional[torch.Tensor] = None):
        B, S = input_ids.shape
        x = self.model.embed_tokens(input_ids)
        cos, sin = self.rope(S, x.device, x.dtype)
        for layer in self.model.layers:
            x = layer(x, cos, sin, keep_mask)
        return self.lm_head(self.model.norm(x))

    def hf_state_dict(self) -> Dict[str, torch.Tensor]:
        return {k: v for k, v in self.state_dict().items()}
