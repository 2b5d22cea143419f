"""Linear-layer GEMMs on the tcgen05 kernel (csrc/kernels/gemm_sm100.cu).

Shapes follow the PyTorch ``F.linear`` convention: ``x [T, K]``, ``w [N, K]``, ``y [T, N]``.

* ``linear_fwd``     y  = x w^T            (both operands K-major)
* ``linear_dgrad``   dx = dy w             (w read MN-major: no transpose copy)
* ``linear_wgrad``   dW (+)= dy^T x        (both read MN-major; fp32 accumulate epilogue)

CPU tensors run the fp32 reference (``torch.matmul``); CUDA tensors always run the kernel.
"""
from __future__ import annotations

from typing import Optional

import torch

from ._ext import kernels

EPI_BF16, EPI_BF16_RESID, EPI_F32, EPI_F32_ACC = 0, 1, 2, 3


def gemm(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, a_mn: bool, b_mn: bool,
         epi: int = EPI_BF16, resid: Optional[torch.Tensor] = None, alpha: float = 1.0,
         bn: int = 0, max_ctas: int = 0) -> torch.Tensor:
    """``out = epi(alpha * op(a) @ op(b))`` with op(a) ``[M, K]`` and op(b) ``[K, N]``."""
    if not a.is_cuda:
        A = (a.t() if a_mn else a).float()
        B = (b if b_mn else b.t()).float()
        r = alpha * (A @ B)
        if epi == EPI_BF16_RESID:
            r = r + resid.float()
        if epi == EPI_F32_ACC:
            out += r
        else:
            out.copy_(r)
        return out
    _check_gemm_operands(a, b, out, b_mn)
    kernels().gemm(a, b, out, a_mn, b_mn, epi, resid, alpha, bn, max_ctas)
    return out


def _check_gemm_operands(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor, b_mn: bool):
    """Shape and alignment rules of the tcgen05 GEMM (TMA rows start on 16 bytes, the epilogue
    stores 32-column chunks), checked before the launch so a bad call raises here."""
    N = b.shape[1] if b_mn else b.shape[0]
    if N % 32:
        raise ValueError(f"gemm: N = {N} is not a multiple of 32")
    for name, t in (("a", a), ("b", b), ("out", out)):
        if t.dim() != 2 or t.stride(1) != 1:
            raise ValueError(f"gemm: {name} must be 2-D with unit column stride")
        if t.data_ptr() % 16:
            raise ValueError(f"gemm: {name} is not 16-byte aligned")
    if a.stride(0) % 8 or b.stride(0) % 8:
        raise ValueError("gemm: row strides of a and b must be multiples of 8 elements")


def linear_fwd(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
               resid: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    return gemm(x, w, out, False, False, EPI_BF16_RESID if resid is not None else EPI_BF16,
                resid)


def linear_fwd_ce(x: torch.Tensor, w: torch.Tensor, labels: torch.Tensor):
    """Per-token cross entropy of ``logits = x w^T`` against ``labels`` (< 0: ignored, loss 0)
    without storing the logits: the GEMM epilogue reduces every 256-column tile of a row to
    (max, sum of exp, label logit) and a combine kernel forms ``lse`` and the loss.
    Returns ``(loss [M], lse [M])`` in fp32."""
    M, N = x.shape[0], w.shape[0]
    f32 = dict(dtype=torch.float32, device=x.device)
    if not x.is_cuda:
        from . import reference as ref
        return ref.cross_entropy(x.float() @ w.float().t(), labels)
    nt = (N + 255) // 256
    pmax = torch.empty(M, nt, **f32)
    psum = torch.empty(M, nt, **f32)
    ptgt = torch.empty(M, **f32)
    loss, lse = torch.empty(M, **f32), torch.empty(M, **f32)
    k = kernels()
    k.gemm_ce_part(x, w, labels, pmax, psum, ptgt)
    k.ce_combine(pmax, psum, ptgt, labels, N, loss, lse)
    return loss, lse


def linear_ce_grad(x: torch.Tensor, w: torch.Tensor, labels: torch.Tensor, lse: torch.Tensor,
                   dloss: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``dlogits = (softmax(x w^T) - onehot(labels)) * dloss`` (bf16 ``[M, N]``) with the logits
    recomputed inside the GEMM (rows with ``labels < 0`` are zero)."""
    M, N = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(M, N, dtype=x.dtype, device=x.device)
    if not x.is_cuda:
        from . import reference as ref
        out.copy_(ref.cross_entropy_bwd(x.float() @ w.float().t(), labels, lse, dloss))
        return out
    kernels().gemm_ce_grad(x, w, labels, lse.contiguous(), dloss.contiguous(), out)
    return out


def linear_fwd_rope(x: torch.Tensor, w: torch.Tensor, pos: torch.Tensor, table: torch.Tensor,
                    rope_cols: int, head_dim: int, out: Optional[torch.Tensor] = None
                    ) -> torch.Tensor:
    """``y = x w^T`` with rotate-half RoPE applied to columns ``[0, rope_cols)`` (heads of
    ``head_dim``) at positions ``pos [T]``, fused into the GEMM epilogue (the q and k heads of a
    fused qkv projection)."""
    if out is None:
        out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
    if not x.is_cuda:
        from . import reference as ref
        y = x.float() @ w.float().t()
        n = rope_cols // head_dim
        q = y[:, :rope_cols].view(-1, n, head_dim)
        y[:, :rope_cols] = ref.rope(q, pos, table).reshape(-1, rope_cols)
        out.copy_(y)
        return out
    kernels().gemm_rope(x, w, out, pos, table, rope_cols, head_dim)
    return out


def linear_fwd_swiglu(x: torch.Tensor, w: torch.Tensor):
    """``gu = x w^T`` for ``w = [gate; up]`` and ``h = silu(gate) * up`` from the same kernel
    (SwiGLU in the GEMM epilogue).  Returns ``(gu [T, 2F], h [T, F])``; ``gu`` is what the
    backward needs."""
    F = w.shape[0] // 2
    gu = torch.empty(x.shape[0], 2 * F, dtype=x.dtype, device=x.device)
    h = torch.empty(x.shape[0], F, dtype=x.dtype, device=x.device)
    if not x.is_cuda or F % 128:
        gu = gemm(x, w, gu, False, False)
        from . import fused
        return gu, fused.swiglu_fwd(gu, out=h)
    kernels().gemm_swiglu(x, w, gu, h)
    return gu, h


def linear_dgrad_swiglu(dy: torch.Tensor, wd: torch.Tensor, gu: torch.Tensor,
                        gu_rows: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``d[gate; up]`` of ``h = silu(gate) * up`` given ``dy`` at the down projection's output:
    ``dh = dy wd`` (``wd [H, F]``) feeds the SwiGLU backward in the GEMM epilogue, with the saved
    ``gu`` rows ``gu_rows`` (kept rows of the forward's ``gu``; all rows when ``None``).
    Returns ``dgu [T, 2F]``; ``dh`` is never materialised."""
    F = wd.shape[1]
    dgu = torch.empty(dy.shape[0], 2 * F, dtype=dy.dtype, device=dy.device)
    if not dy.is_cuda:
        from . import fused
        dh = (dy.float() @ wd.float()).to(dy.dtype)
        return fused.swiglu_bwd(dh, gu, gu_rows, out=dgu)
    if F % 32:
        raise ValueError(f"linear_dgrad_swiglu: F = {F} is not a multiple of 32")
    kernels().gemm_swiglu_bwd(dy, wd, gu, gu_rows, dgu)
    return dgu


def linear_dgrad(dy: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None,
                 resid: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(dy.shape[0], w.shape[1], dtype=dy.dtype, device=dy.device)
    return gemm(dy, w, out, False, True, EPI_BF16_RESID if resid is not None else EPI_BF16,
                resid)


def linear_wgrad(dy: torch.Tensor, x: torch.Tensor, dw: torch.Tensor,
                 accumulate: bool = True, alpha: float = 1.0) -> torch.Tensor:
    """``dw (+)= alpha * dy^T x``; ``dw`` is fp32 ``[N, K]`` (the flat gradient bucket)."""
    return gemm(dy, x, dw, True, True, EPI_F32_ACC if accumulate else EPI_F32, None, alpha)
