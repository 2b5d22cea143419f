"""Python entry points of the fused sm_100a kernels.

Every function takes preallocated outputs where the training step reuses buffers.  CUDA tensors
go to the compiled kernels (``centrifuge_b200._kernels``); CPU tensors run the fp32 definitions
in :mod:`centrifuge_b200.ops.reference`.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import reference as ref
from ._ext import kernels


# ---------------------------------------------------------------- RMSNorm
def rmsnorm_fwd(x: torch.Tensor, w: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None,
                rstd: Optional[torch.Tensor] = None):
    if out is None:
        out = torch.empty_like(x)
    if rstd is None:
        rstd = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    if not x.is_cuda:
        y, r = ref.rmsnorm(x, w, eps)
        out.copy_(y)
        rstd.copy_(r)
        return out, rstd
    kernels().rmsnorm_fwd(x, w, out, rstd, eps)
    return out, rstd


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, rstd: torch.Tensor, w: torch.Tensor,
                dw_acc: torch.Tensor, x_rows: Optional[torch.Tensor] = None,
                dres: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None):
    """``dx = dres + d(rmsnorm)/dx`` on the rows ``x[x_rows]``; ``dw_acc += dgamma`` (fp32)."""
    if out is None:
        out = torch.empty_like(dy)
    if not dy.is_cuda:
        xs = x if x_rows is None else x[x_rows.long()]
        rs = rstd if x_rows is None else rstd[x_rows.long()]
        dx, dw = ref.rmsnorm_bwd(dy, xs, rs, w, dres)
        out.copy_(dx)
        dw_acc += dw
        return out
    partial_rows = max(1, min(dy.shape[0], 148 * 2))
    kernels().rmsnorm_bwd(dy, x, x_rows, rstd, w, dres, out, dw_acc, partial_rows)
    return out


# ---------------------------------------------------------------- RoPE
def rope_(qkv: torch.Tensor, pos: torch.Tensor, n_heads: int, head_dim: int,
          table: torch.Tensor, inverse: bool = False) -> torch.Tensor:
    """In-place RoPE on heads ``[0, n_heads)`` of each ``qkv`` row at positions ``pos``."""
    if not qkv.is_cuda:
        rows = qkv.shape[0]
        view = qkv[:, : n_heads * head_dim].view(rows, n_heads, head_dim)
        view.copy_(ref.rope(view, pos, table, inverse))
        return qkv
    kernels().rope(qkv, pos, n_heads, head_dim, table, inverse)
    return qkv


# ---------------------------------------------------------------- SwiGLU
def swiglu_fwd(gu: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    F = gu.shape[1] // 2
    if out is None:
        out = torch.empty(gu.shape[0], F, dtype=gu.dtype, device=gu.device)
    if not gu.is_cuda:
        out.copy_(ref.swiglu(gu))
        return out
    kernels().swiglu_fwd(gu, out)
    return out


def swiglu_bwd(dh: torch.Tensor, gu: torch.Tensor, gu_rows: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None,
               h_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``d[gate; up]`` from ``dh`` and the saved ``gu`` rows ``gu_rows``.  With ``h_out``
    (``[rows, F]``) the same pass also writes ``h = silu(gate) * up`` of those rows, i.e. the
    forward activation of the kept rows, recomputed instead of gathered."""
    if out is None:
        out = torch.empty(dh.shape[0], 2 * dh.shape[1], dtype=dh.dtype, device=dh.device)
    if not dh.is_cuda:
        g = gu if gu_rows is None else gu[gu_rows.long()]
        out.copy_(ref.swiglu_bwd(dh, g))
        if h_out is not None:
            h_out.copy_(ref.swiglu(g.float()))
        return out
    kernels().swiglu_bwd(dh, gu, gu_rows, out, h_out)
    return out


# ---------------------------------------------------------------- gathers / embedding
def gather_rows(src: torch.Tensor, idx: torch.Tensor, out: Optional[torch.Tensor] = None):
    if out is None:
        out = torch.empty(idx.numel(), src.shape[1], dtype=src.dtype, device=src.device)
    if not src.is_cuda:
        out.copy_(src[idx.long()])
        return out
    kernels().gather_rows(src, idx, out)
    return out


def embedding_fwd(table: torch.Tensor, ids: torch.Tensor, out: Optional[torch.Tensor] = None):
    ids = ids.reshape(-1)
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    if not table.is_cuda:
        out.copy_(table[ids])
        return out
    kernels().embedding_fwd(table, ids.contiguous(), out)
    return out


def embedding_bwd(dy: torch.Tensor, ids: torch.Tensor, dtable: torch.Tensor,
                  id_rows: Optional[torch.Tensor] = None, deterministic: bool = True):
    """``dtable[ids[id_rows[r]]] += dy[r]``.  ``deterministic``: rows are sorted by token and
    each token's rows are summed in row order by one warp (same bits on every run); otherwise
    fp32 atomics, whose summation order varies from run to run."""
    ids = ids.reshape(-1)
    if not dy.is_cuda:
        sel = ids if id_rows is None else ids[id_rows.long()]
        dtable.index_add_(0, sel, dy.float())
        return dtable
    kernels().embedding_bwd(dy, ids.contiguous(), id_rows, dtable, deterministic)
    return dtable


# ---------------------------------------------------------------- cross entropy
def ce_fwd(logits: torch.Tensor, labels: torch.Tensor, loss: Optional[torch.Tensor] = None,
           lse: Optional[torch.Tensor] = None):
    rows = logits.shape[0]
    if loss is None:
        loss = torch.empty(rows, dtype=torch.float32, device=logits.device)
    if lse is None:
        lse = torch.empty(rows, dtype=torch.float32, device=logits.device)
    if not logits.is_cuda:
        l, s = ref.cross_entropy(logits, labels)
        loss.copy_(l)
        lse.copy_(s)
        return loss, lse
    kernels().ce_fwd(logits, labels, loss, lse)
    return loss, lse


def ce_bwd(logits: torch.Tensor, labels: torch.Tensor, lse: torch.Tensor, dloss: torch.Tensor,
           rows: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
           vocab_start: int = 0):
    """dlogits of the rows ``rows`` (all when None); with a vocabulary shard the logits'
    columns are the global ids ``vocab_start + j`` and ``lse`` is the full-vocabulary lse."""
    n = dloss.numel()
    if out is None:
        out = torch.empty(n, logits.shape[1], dtype=logits.dtype, device=logits.device)
    if not logits.is_cuda:
        r = torch.arange(logits.shape[0]) if rows is None else rows.long()
        lab = labels[r]
        V = logits.shape[1]
        p = torch.exp(logits[r].float() - lse[r].unsqueeze(-1))
        loc = lab - vocab_start
        hit = (lab >= 0) & (loc >= 0) & (loc < V)
        p[hit, loc[hit]] -= 1.0
        p = p * dloss.unsqueeze(-1)
        p[lab < 0] = 0
        out.copy_(p)
        return out
    kernels().ce_bwd(logits, rows, labels, lse, dloss, out, vocab_start)
    return out


def ce_partial(logits: torch.Tensor, labels: torch.Tensor, vocab_start: int, out=None):
    """Per-row (max, sum exp(logit - max), label logit or 0) of one vocabulary shard;
    ``out``: three fp32 ``[rows]`` tensors to write them into."""
    rows = logits.shape[0]
    f32 = dict(dtype=torch.float32, device=logits.device)
    pmax, psum, ptgt = out if out is not None else (torch.empty(rows, **f32) for _ in range(3))
    if not logits.is_cuda:
        lf = logits.float()
        pmax.copy_(lf.max(-1).values)
        psum.copy_(torch.exp(lf - pmax.unsqueeze(-1)).sum(-1))
        loc = labels - vocab_start
        hit = (labels >= 0) & (loc >= 0) & (loc < lf.shape[1])
        t = torch.zeros(rows, **f32)
        t[hit] = lf[hit, loc[hit]]
        ptgt.copy_(t)
        return pmax, psum, ptgt
    kernels().ce_partial(logits, labels, pmax, psum, ptgt, vocab_start)
    return pmax, psum, ptgt


# ---------------------------------------------------------------- optimizer
def adamw_(master, grad, m, v, param, lr, beta1, beta2, eps, wd, step, grad_scale=None):
    """Fused AdamW step on flat fp32 buffers; writes the bf16 copy into ``param``."""
    bc1 = 1.0 - beta1 ** step
    bc2 = 1.0 - beta2 ** step
    if not master.is_cuda:
        g = grad * (grad_scale if grad_scale is not None else 1.0)
        master.mul_(1 - lr * wd)
        m.mul_(beta1).add_(g, alpha=1 - beta1)
        v.mul_(beta2).addcmul_(g, g, value=1 - beta2)
        denom = (v.sqrt() / math.sqrt(bc2)).add_(eps)
        master.addcdiv_(m, denom, value=-lr / bc1)
        param.copy_(master)
        return
    kernels().adamw(master, grad, m, v, param, lr, beta1, beta2, eps, wd, bc1, bc2, grad_scale)


def grad_norm_clip_coef(grad: torch.Tensor, max_norm: float, extra_scale: float,
                        coef: torch.Tensor, norm: torch.Tensor,
                        partial: Optional[torch.Tensor] = None,
                        extra_sumsq: Optional[torch.Tensor] = None):
    """On-device ``coef = clip(max_norm / ||g * extra_scale||) * extra_scale``.

    ``extra_sumsq`` lets data-parallel ranks add the squared norms of the other shards (it is
    the all-reduced sum of the per-rank partial sums).
    """
    if not grad.is_cuda:
        s = grad.float().pow(2).sum()
        if extra_sumsq is not None:
            s = extra_sumsq.sum()
        n = s.sqrt() * extra_scale
        c = 1.0
        if max_norm > 0 and n > max_norm:
            c = max_norm / (float(n) + 1e-6)
        coef.fill_(c * extra_scale)
        norm.fill_(float(n))
        return coef
    k = kernels()
    if extra_sumsq is None:
        if partial is None:
            partial = torch.empty(148 * 4, dtype=torch.float32, device=grad.device)
        k.sumsq(grad, partial)
        extra_sumsq = partial
    k.clip_coef(extra_sumsq, max_norm, extra_scale, coef, norm)
    return coef


# ---------------------------------------------------------------- attention
def attn_fwd(qkv: torch.Tensor, B: int, S: int, nh: int, nkv: int, hd: int,
             out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
             scale: Optional[float] = None):
    """Causal GQA attention over the fused ``qkv [B*S, (nh+2nkv)*hd]`` rows.

    Returns ``o [B*S, nh*hd]`` (bf16) and ``lse [B*S, nh]`` (fp32).
    """
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    T = B * S
    if out is None:
        out = torch.empty(T, nh * hd, dtype=qkv.dtype, device=qkv.device)
    if lse is None:
        lse = torch.empty(T, nh, dtype=torch.float32, device=qkv.device)
    if not qkv.is_cuda:
        q = qkv[:, : nh * hd].reshape(B, S, nh, hd)
        k = qkv[:, nh * hd:(nh + nkv) * hd].reshape(B, S, nkv, hd)
        v = qkv[:, (nh + nkv) * hd:(nh + 2 * nkv) * hd].reshape(B, S, nkv, hd)
        o, l = ref.attention(q, k, v, True, scale)
        out.copy_(o.reshape(T, nh * hd))
        lse.copy_(l.reshape(T, nh))
        return out, lse
    kernels().attn_fwd(qkv, out, lse, B, S, nh, nkv, hd, scale)
    return out, lse


def attn_bwd(qkv_k: torch.Tensor, qkv_full: torch.Tensor, o_k: torch.Tensor, do_k: torch.Tensor,
             lse_k: torch.Tensor, pos_k: torch.Tensor, B: int, S: int, Sk: int, nh: int,
             nkv: int, hd: int, dqkv_k: Optional[torch.Tensor] = None,
             scale: Optional[float] = None,
             rope_table: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Filtered (restore-Q) attention backward; returns ``dqkv_k [B*Sk, ld]``.

    With ``rope_table`` the q and k gradients come out with the RoPE backward applied (rotated
    back to the pre-RoPE projection outputs at the kept rows' positions)."""
    scale = scale if scale is not None else 1.0 / math.sqrt(hd)
    if dqkv_k is None:
        dqkv_k = torch.empty_like(qkv_k)
    if not qkv_k.is_cuda:
        q = qkv_k[:, : nh * hd].reshape(B, Sk, nh, hd)
        k = qkv_full[:, nh * hd:(nh + nkv) * hd].reshape(B, S, nkv, hd)
        v = qkv_full[:, (nh + nkv) * hd:(nh + 2 * nkv) * hd].reshape(B, S, nkv, hd)
        dq, dk, dv = ref.attention_bwd_filtered(
            q, k, v, o_k.reshape(B, Sk, nh, hd), do_k.reshape(B, Sk, nh, hd),
            lse_k.reshape(B, Sk, nh), pos_k.reshape(B, Sk), scale)
        dq = dq.reshape(B * Sk, nh, hd)
        dk = dk.reshape(B * Sk, nkv, hd)
        if rope_table is not None:
            pf = pos_k.reshape(-1)
            dq = ref.rope(dq, pf, rope_table, inverse=True)
            dk = ref.rope(dk, pf, rope_table, inverse=True)
        dqkv_k[:, : nh * hd] = dq.reshape(B * Sk, nh * hd)
        dqkv_k[:, nh * hd:(nh + nkv) * hd] = dk.reshape(B * Sk, nkv * hd)
        dqkv_k[:, (nh + nkv) * hd:(nh + 2 * nkv) * hd] = dv.reshape(B * Sk, nkv * hd)
        return dqkv_k
    delta = torch.empty(B * Sk * nh, dtype=torch.float32, device=qkv_k.device)
    kernels().attn_bwd(qkv_k, qkv_full, o_k, do_k, lse_k, pos_k, dqkv_k, delta, B, S, Sk, nh, nkv,
                       hd, scale, rope_table)
    return dqkv_k
    delta = torch.empty(B * Sk * nh, dtype=torch.float32, device=qkv_k.device)
    kernels().attn_bwd(qkv_k, qkv_full, o_k, do_k, lse_k, pos_k, dqkv_k, delta, B, S, Sk, nh, nkv,
                       hd, scale)
    return dqkv_k
