"""CPU checks of the fp32 op definitions that serve as kernel oracles."""
import torch

from centrifuge_b200.ops import fused, reference as ref


def test_filtered_attention_bwd_matches_detached_kv_autograd():
    torch.manual_seed(0)
    B, S, nh, nkv, hd = 2, 24, 4, 2, 8
    q = torch.randn(B, S, nh, hd, requires_grad=True)
    k = torch.randn(B, S, nkv, hd, requires_grad=True)
    v = torch.randn(B, S, nkv, hd, requires_grad=True)
    keep = torch.rand(B, S) < 0.5
    keep[:, -1] = True
    Sk = int(keep.sum(1).min())
    for b in range(B):  # equal kept count per row
        idx = keep[b].nonzero().squeeze(-1)
        keep[b, idx[: len(idx) - Sk]] = False
    kd = torch.where(keep.view(B, S, 1, 1), k, k.detach())
    vd = torch.where(keep.view(B, S, 1, 1), v, v.detach())
    o, lse = ref.attention(q, kd, vd)
    pos = keep.nonzero()[:, 1].view(B, Sk)
    do = torch.randn(B, Sk, nh, hd)
    o_k = torch.stack([o[b, pos[b]] for b in range(B)])
    (o_k * do).sum().backward()
    q_k = torch.stack([q[b, pos[b]] for b in range(B)]).detach()
    lse_k = torch.stack([lse[b, pos[b]] for b in range(B)]).detach()
    dq, dk, dv = ref.attention_bwd_filtered(q_k, k.detach(), v.detach(), o_k.detach(), do, lse_k, pos)
    for b in range(B):
        assert torch.allclose(dq[b], q.grad[b, pos[b]], atol=1e-5)
        assert torch.allclose(dk[b], k.grad[b, pos[b]], atol=1e-5)
        assert torch.allclose(dv[b], v.grad[b, pos[b]], atol=1e-5)
    # dropped rows get no gradient at all
    assert torch.all(q.grad[~keep] == 0) and torch.all(k.grad[~keep] == 0)


def test_fused_cpu_paths_roundtrip():
    torch.manual_seed(1)
    B, S, nh, nkv, hd = 1, 16, 2, 1, 8
    qkv = torch.randn(B * S, (nh + 2 * nkv) * hd)
    o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd)
    pos = torch.arange(S, dtype=torch.int32).view(1, S)
    d = fused.attn_bwd(qkv, qkv, o, torch.randn_like(o), lse, pos, B, S, S, nh, nkv, hd)
    assert d.shape == qkv.shape and torch.isfinite(d).all()
