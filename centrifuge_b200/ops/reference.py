"""Plain-PyTorch fp32 definitions of every fused op.

These are the numerical oracles the sm_100a kernels are tested against, and the code path the
ops take on CPU tensors (unit tests and the CPU filtered-gradient oracle run here).
"""
from __future__ import annotations

import math
from typing import Optional

import torch


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float):
    xf = x.float()
    rstd = torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (xf * rstd * w.float()), rstd.squeeze(-1)


def rmsnorm_bwd(dy, x, rstd, w, dres=None):
    dyf, xf, wf = dy.float(), x.float(), w.float()
    r = rstd.float().unsqueeze(-1)
    H = x.shape[-1]
    dot = (wf * dyf * xf).sum(-1, keepdim=True)
    dx = r * wf * dyf - xf * dot * r.pow(3) / H
    if dres is not None:
        dx = dx + dres.float()
    dw = (dyf * xf * r).sum(0)
    return dx, dw


def rope_table(max_pos: int, head_dim: int, theta: float, device=None) -> torch.Tensor:
    """``[max_pos, head_dim/2, 2]`` fp32 (cos, sin) of ``pos * theta^(-2i/d)`` (HF convention)."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    pos = torch.arange(max_pos, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    return torch.stack([freqs.cos(), freqs.sin()], dim=-1).contiguous().to(device)


def rope(x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor, inverse: bool = False):
    """Rotate-half RoPE of ``x [rows, n_heads, hd]`` at positions ``pos [rows]``."""
    hd = x.shape[-1]
    half = hd // 2
    cs = table[pos.long()]  # [rows, half, 2]
    c = cs[..., 0].unsqueeze(1)
    s = cs[..., 1].unsqueeze(1)
    if inverse:
        s = -s
    x1, x2 = x[..., :half].float(), x[..., half:].float()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1)


def swiglu(gu: torch.Tensor):
    F = gu.shape[-1] // 2
    g, u = gu[..., :F].float(), gu[..., F:].float()
    return torch.nn.functional.silu(g) * u


def swiglu_bwd(dh, gu):
    F = gu.shape[-1] // 2
    g, u, d = gu[..., :F].float(), gu[..., F:].float(), dh.float()
    s = torch.sigmoid(g)
    du = d * g * s
    dg = d * u * s * (1 + g * (1 - s))
    return torch.cat([dg, du], dim=-1)


def cross_entropy(logits: torch.Tensor, labels: torch.Tensor):
    lf = logits.float()
    lse = torch.logsumexp(lf, dim=-1)
    safe = labels.clamp(min=0)
    loss = lse - lf.gather(-1, safe.unsqueeze(-1)).squeeze(-1)
    loss = torch.where(labels >= 0, loss, torch.zeros_like(loss))
    return loss, lse


def cross_entropy_bwd(logits, labels, lse, dloss):
    p = torch.exp(logits.float() - lse.unsqueeze(-1))
    onehot = torch.zeros_like(p)
    valid = labels >= 0
    onehot[valid, labels[valid]] = 1.0
    g = (p - onehot) * dloss.unsqueeze(-1)
    g[~valid] = 0
    return g


def attention(q, k, v, causal: bool = True, scale: Optional[float] = None):
    """``q [B, S, nh, hd]``, ``k, v [B, S, nkv, hd]`` -> ``(o [B, S, nh, hd], lse [B, S, nh])``."""
    B, S, nh, hd = q.shape
    nkv = k.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    rep = nh // nkv
    kf = k.float().repeat_interleave(rep, dim=2)
    vf = v.float().repeat_interleave(rep, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", q.float(), kf) * scale
    if causal:
        m = torch.ones(S, S, dtype=torch.bool, device=q.device).triu(1)
        s = s.masked_fill(m, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)  # [B, nh, S]
    p = torch.exp(s - lse.unsqueeze(-1))
    o = torch.einsum("bhqk,bkhd->bqhd", p, vf)
    return o, lse.permute(0, 2, 1)


def attention_bwd_filtered(q_k, k_full, v_full, o_k, do_k, lse_k, pos_k, scale=None):
    """Restore-Q filtered attention backward (fp32).

    ``q_k/o_k/do_k [B, Sk, nh, hd]`` are the kept query rows, ``k_full/v_full [B, S, nkv, hd]``
    every key, ``lse_k [B, Sk, nh]``, ``pos_k [B, Sk]`` the kept positions.  Returns
    ``dq_k [B, Sk, nh, hd]`` (all keys contribute) and ``dk_k, dv_k [B, Sk, nkv, hd]``
    (kept keys, kept queries only).
    """
    B, Sk, nh, hd = q_k.shape
    S, nkv = k_full.shape[1], k_full.shape[2]
    rep = nh // nkv
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    kf = k_full.float().repeat_interleave(rep, dim=2)
    vf = v_full.float().repeat_interleave(rep, dim=2)
    qf, of, dof = q_k.float(), o_k.float(), do_k.float()
    s = torch.einsum("bqhd,bkhd->bhqk", qf, kf) * scale  # [B, nh, Sk, S]
    keys = torch.arange(S, device=q_k.device)
    valid = keys.view(1, 1, S) <= pos_k.long().view(B, Sk, 1)  # [B, Sk, S]
    p = torch.exp(s - lse_k.float().permute(0, 2, 1).unsqueeze(-1))
    p = torch.where(valid.unsqueeze(1), p, torch.zeros_like(p))
    dp = torch.einsum("bqhd,bkhd->bhqk", dof, vf)
    delta = (dof * of).sum(-1).permute(0, 2, 1).unsqueeze(-1)  # [B, nh, Sk, 1]
    ds = p * (dp - delta)
    dq = torch.einsum("bhqk,bkhd->bqhd", ds, kf) * scale
    # kept keys only: gather key columns at the kept positions
    idx = pos_k.long().view(B, 1, 1, Sk).expand(B, nh, Sk, Sk)
    ds_kk = torch.gather(ds, 3, idx)  # [B, nh, Sk(q), Sk(k)]
    p_kk = torch.gather(p, 3, idx)
    dk = torch.einsum("bhqk,bqhd->bkhd", ds_kk, qf) * scale
    dv = torch.einsum("bhqk,bqhd->bkhd", p_kk, dof)
    dk = dk.view(B, Sk, nkv, rep, hd).sum(3)
    dv = dv.view(B, Sk, nkv, rep, hd).sum(3)
    return dq, dk, dv
