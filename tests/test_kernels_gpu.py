"""sm_100a kernels against plain-PyTorch fp32 definitions of the same ops."""
import math

import pytest
import torch

from centrifuge_b200.ops import fused, gemm, reference as ref, select

pytestmark = pytest.mark.gpu
dev = "cuda"


def rel_err(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (304, 512, 200), (1024, 2560, 2048),
                                   (80, 96, 136)])
@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("bn", [128, 256, 512])  # 512: 256 x 256 tile on a CTA pair
def test_gemm_layouts(M, N, K, a_mn, b_mn, bn):
    torch.manual_seed(0)
    A = torch.randn(M, K, device=dev).bfloat16()
    Bm = torch.randn(K, N, device=dev).bfloat16()
    a = A.t().contiguous() if a_mn else A
    b = Bm.contiguous() if b_mn else Bm.t().contiguous()
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    gemm.gemm(a, b, out, a_mn, b_mn, gemm.EPI_BF16, bn=bn)
    torch.cuda.synchronize()
    want = A.float() @ Bm.float()
    assert rel_err(out, want) < 1e-2
    from centrifuge_b200.ops import kernels
    assert kernels().gemm_error_word(0, True) == 0


@pytest.mark.parametrize("M,N,K", [(512, 768, 384), (4096, 2048, 1024), (300, 1000 - 8, 544)])
def test_gemm_epilogues(M, N, K):
    torch.manual_seed(1)
    x = torch.randn(M, K, device=dev).bfloat16()
    w = torch.randn(N, K, device=dev).bfloat16()
    r = torch.randn(M, N, device=dev).bfloat16()
    y = gemm.linear_fwd(x, w, resid=r)
    assert rel_err(y, x.float() @ w.float().t() + r.float()) < 1e-2
    dy = torch.randn(M, N, device=dev).bfloat16()
    dx = gemm.linear_dgrad(dy, w)
    assert rel_err(dx, dy.float() @ w.float()) < 1e-2
    dw = torch.ones(N, K, device=dev)
    gemm.linear_wgrad(dy, x, dw, accumulate=True)
    assert rel_err(dw, 1 + dy.float().t() @ x.float()) < 1e-2
    gemm.linear_wgrad(dy, x, dw, accumulate=False, alpha=0.5)
    assert rel_err(dw, 0.5 * dy.float().t() @ x.float()) < 1e-2


@pytest.mark.parametrize("M,H,F,gathered", [(4096, 2048, 5632, True), (1000, 512, 1024, False),
                                            (300, 256, 96, True)])
def test_gemm_swiglu_bwd_epilogue(M, H, F, gathered):
    """Down-projection dgrad with the SwiGLU backward in the epilogue vs the fp32 oracle."""
    torch.manual_seed(15)
    dy = torch.randn(M, H, device=dev).bfloat16()
    wd = (torch.randn(H, F, device=dev) / H ** 0.5).bfloat16()
    T = 2 * M if gathered else M
    gu = (2 * torch.randn(T, 2 * F, device=dev)).bfloat16()
    rows = (torch.randperm(T, device=dev)[:M].sort().values.int() if gathered else None)
    dgu = gemm.linear_dgrad_swiglu(dy, wd, gu, rows)
    torch.cuda.synchronize()
    dh = dy.float() @ wd.float()
    g_rows = gu[rows.long()] if gathered else gu
    want = ref.swiglu_bwd(dh, g_rows.float())
    assert rel_err(dgu, want) < 1e-2
    from centrifuge_b200.ops import kernels
    assert kernels().gemm_error_word(0, True) == 0


def test_gemm_rejects_unsupported_shapes():
    x = torch.randn(64, 520, device=dev).bfloat16()
    w = torch.randn(96, 520, device=dev).bfloat16()
    with pytest.raises(ValueError):
        gemm.linear_dgrad(torch.randn(64, 96, device=dev).bfloat16(), w)  # N = 520
    with pytest.raises(ValueError):
        gemm.linear_fwd(x[:, 1:513], w[:, :512])  # a not 16-byte aligned


@pytest.mark.parametrize("M,N,K", [(2560, 2048, 8192), (2048, 5632, 4096), (768, 4096, 6000)])
def test_gemm_wgrad_split_k(M, N, K):
    """Weight-gradient shapes whose tile count leaves the last wave mostly empty run split-K
    (fp32 partial sums reduced into dW); the result must match the fp32 oracle."""
    torch.manual_seed(5)
    dy = torch.randn(K, M, device=dev).bfloat16()
    x = torch.randn(K, N, device=dev).bfloat16()
    dw0 = torch.randn(M, N, device=dev)
    dw = dw0.clone()
    gemm.linear_wgrad(dy, x, dw, accumulate=True)
    torch.cuda.synchronize()
    want = dw0 + dy.float().t() @ x.float()
    assert rel_err(dw, want) < 2e-3
    from centrifuge_b200.ops import kernels
    assert kernels().gemm_error_word(0, True) == 0


@pytest.mark.parametrize("T,H,Tk", [(300, 2048, 100), (9000, 2048, 4500), (3000, 4096, 1200),
                                   (500, 1000, 250), (700, 768, 700)])
def test_rmsnorm(T, H, Tk):
    torch.manual_seed(2)
    x = torch.randn(T, H, device=dev).bfloat16()
    w = (1 + 0.1 * torch.randn(H, device=dev)).bfloat16()
    y, rstd = fused.rmsnorm_fwd(x, w, 1e-5)
    yr, rr = ref.rmsnorm(x, w, 1e-5)
    assert rel_err(y, yr) < 1e-2 and rel_err(rstd, rr) < 1e-4
    rows = torch.randperm(T, device=dev)[:Tk].sort().values.int()
    dy = torch.randn(Tk, H, device=dev).bfloat16()
    dres = torch.randn(Tk, H, device=dev).bfloat16()
    dw = torch.zeros(H, device=dev)
    dx = fused.rmsnorm_bwd(dy, x, rstd, w, dw, x_rows=rows, dres=dres)
    dxr, dwr = ref.rmsnorm_bwd(dy, x[rows.long()], rstd[rows.long()], w, dres)
    assert rel_err(dx, dxr) < 1e-2 and rel_err(dw, dwr) < 1e-3


def test_rope_roundtrip():
    torch.manual_seed(3)
    T, nh, nkv, hd = 64, 4, 2, 64
    table = ref.rope_table(128, hd, 10000.0, dev)
    qkv = torch.randn(T, (nh + 2 * nkv) * hd, device=dev).bfloat16()
    pos = torch.randint(0, 128, (T,), device=dev, dtype=torch.int32)
    want = ref.rope(qkv[:, : (nh + nkv) * hd].view(T, nh + nkv, hd), pos, table)
    out = qkv.clone()
    fused.rope_(out, pos, nh + nkv, hd, table)
    assert rel_err(out[:, : (nh + nkv) * hd].view(T, nh + nkv, hd), want) < 1e-2
    assert torch.equal(out[:, (nh + nkv) * hd:], qkv[:, (nh + nkv) * hd:])
    fused.rope_(out, pos, nh + nkv, hd, table, inverse=True)
    assert rel_err(out, qkv) < 2e-2


def test_swiglu():
    torch.manual_seed(4)
    T, F = 100, 512
    gu = torch.randn(T, 2 * F, device=dev).bfloat16()
    h = fused.swiglu_fwd(gu)
    assert rel_err(h, ref.swiglu(gu)) < 1e-2
    rows = torch.arange(0, T, 3, device=dev, dtype=torch.int32)
    dh = torch.randn(rows.numel(), F, device=dev).bfloat16()
    dgu = fused.swiglu_bwd(dh, gu, rows)
    assert rel_err(dgu, ref.swiglu_bwd(dh, gu[rows.long()])) < 1e-2
    # the kept rows' h recomputed in the backward pass equals the forward's h bit for bit
    h_k = torch.empty_like(dh)
    dgu2 = fused.swiglu_bwd(dh, gu, rows, h_out=h_k)
    assert torch.equal(dgu2, dgu)
    assert torch.equal(h_k, h[rows.long()])
    if F % 128 == 0:  # and equals the h of the SwiGLU GEMM epilogue
        x = torch.randn(T, 256, device=dev).bfloat16()
        w = (torch.randn(2 * F, 256, device=dev) / 16).bfloat16()
        gu_g, h_g = gemm.linear_fwd_swiglu(x, w)
        h_k2 = torch.empty_like(dh)
        fused.swiglu_bwd(dh, gu_g, rows, h_out=h_k2)
        assert torch.equal(h_k2, h_g[rows.long()])


def test_gather_embedding():
    torch.manual_seed(5)
    V, H, T = 1000, 256, 64
    table = torch.randn(V, H, device=dev).bfloat16()
    ids = torch.randint(0, V, (T,), device=dev)
    e = fused.embedding_fwd(table, ids)
    assert torch.equal(e, table[ids])
    idx = torch.tensor([3, 5, 7, 63], device=dev, dtype=torch.int32)
    g = fused.gather_rows(e, idx)
    assert torch.equal(g, e[idx.long()])
    dt = torch.zeros(V, H, device=dev)
    dy = torch.randn(4, H, device=dev).bfloat16()
    fused.embedding_bwd(dy, ids, dt, idx)
    want = torch.zeros(V, H, device=dev).index_add_(0, ids[idx.long()], dy.float())
    assert rel_err(dt, want) < 1e-5



def test_embedding_bwd_deterministic():
    """Sorted-run embedding gradient: matches the fp32 scatter-add, repeated tokens included,
    and gives the same bits on every call (the atomic variant does not promise that)."""
    torch.manual_seed(15)
    V, H, T, R = 50, 2048, 4096, 3000
    ids = torch.randint(0, V, (T,), device=dev)  # ~60 rows per token: long runs
    rows = torch.randperm(T, device=dev)[:R].sort().values.int()
    dy = torch.randn(R, H, device=dev).bfloat16()
    base = torch.randn(V, H, device=dev)
    want = base.clone().index_add_(0, ids[rows.long()], dy.float())
    outs = []
    for _ in range(2):
        dt = base.clone()
        fused.embedding_bwd(dy, ids, dt, rows, deterministic=True)
        outs.append(dt)
    assert rel_err(outs[0], want) < 1e-6
    assert torch.equal(outs[0], outs[1])
    dt = base.clone()
    fused.embedding_bwd(dy, ids, dt, rows, deterministic=False)
    assert rel_err(dt, want) < 1e-6
    # without a row map
    dt = base.clone()
    fused.embedding_bwd(dy, ids[:R], dt)
    assert rel_err(dt, base.clone().index_add_(0, ids[:R], dy.float())) < 1e-6


def test_ex2_poly_accuracy():
    """The attention forward's FMA-pipe exponential: relative error within 1e-4 of 2^x over the
    range the softmax uses ([-125, 8]), exactly the powers of two at integers, 2^-125 at most
    for masked (-inf) scores."""
    from centrifuge_b200.ops import kernels
    x = torch.cat([torch.linspace(-125.0, 8.0, 1 << 20, device=dev),
                   torch.arange(-30, 9, device=dev, dtype=torch.float32)])
    y = torch.empty_like(x)
    kernels().ex2_poly(x, y)
    want = torch.exp2(x.double())
    rel = ((y.double() - want).abs() / want).max().item()
    assert rel < 1e-4, rel
    # MUFU ex2.approx is specified to about 2 ulp; the polynomial's 7.5e-5 is far below the
    # bf16 rounding (2^-9) that P goes through
    z = torch.tensor([-float("inf"), -1000.0], device=dev)
    w = torch.empty_like(z)
    kernels().ex2_poly(z, w)
    assert (w >= 0).all() and (w <= 2.0 ** -124).all()

def test_cross_entropy():
    torch.manual_seed(6)
    T, V = 64, 32000
    logits = (3 * torch.randn(T, V, device=dev)).bfloat16()
    labels = torch.randint(0, V, (T,), device=dev)
    labels[5] = -100
    loss, lse = fused.ce_fwd(logits, labels)
    lr, sr = ref.cross_entropy(logits, labels)
    assert rel_err(loss, lr) < 1e-4 and rel_err(lse, sr) < 1e-5
    rows = torch.tensor([0, 5, 9, 63], device=dev, dtype=torch.int32)
    dloss = torch.rand(4, device=dev)
    g = fused.ce_bwd(logits, labels, lse, dloss, rows)
    want = ref.cross_entropy_bwd(logits[rows.long()], labels[rows.long()], sr[rows.long()], dloss)
    assert rel_err(g, want) < 1e-2


def test_adamw_matches_torch():
    torch.manual_seed(7)
    n = 10003
    p = torch.randn(n, device=dev)
    g = torch.randn(n, device=dev)
    m = torch.zeros(n, device=dev)
    v = torch.zeros(n, device=dev)
    pb = torch.empty(n, device=dev, dtype=torch.bfloat16)
    tp = torch.nn.Parameter(p.clone())
    opt = torch.optim.AdamW([tp], lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1)
    for step in range(1, 4):
        tp.grad = g.clone()
        opt.step()
        fused.adamw_(p, g, m, v, pb, 1e-3, 0.9, 0.95, 1e-8, 0.1, step)
    assert rel_err(p, tp.detach()) < 1e-5
    assert rel_err(pb, tp.detach()) < 1e-2


def test_clip_coef():
    g = torch.full((1000,), 2.0, device=dev)
    coef = torch.empty(1, device=dev)
    norm = torch.empty(1, device=dev)
    fused.grad_norm_clip_coef(g, 1.0, 0.5, coef, norm)
    n = math.sqrt(1000 * 4.0) * 0.5
    assert abs(norm.item() - n) < 1e-3
    assert abs(coef.item() - 0.5 / (n + 1e-6)) < 1e-6


@pytest.mark.parametrize("S,drop", [(2048, 0.5), (224, 0.5), (4096, 0.3)])
def test_drop_smallest_and_keep_index(S, drop):
    from centrifuge_b200.loss import num_dropped
    torch.manual_seed(8)
    B = 3
    score = torch.randn(B, S - 1, device=dev)
    k = num_dropped(S, drop)
    mask = torch.ones(B, S, dtype=torch.long, device=dev)
    select.drop_smallest_(score, mask, k, 0, S - 1)
    want = torch.ones(B, S, dtype=torch.long)
    _, idx = torch.topk(score.cpu(), k, dim=1, largest=False)
    want.scatter_(1, idx, 0)
    assert torch.equal(mask.cpu(), want)
    pos, flat, err = select.keep_index(mask, S - k)
    assert int(err[0]) == 0
    pos_c, flat_c, _ = select.keep_index(want, S - k)
    assert torch.equal(pos.cpu(), pos_c) and torch.equal(flat.cpu(), flat_c)


@pytest.mark.parametrize("left", [True, False])
def test_token_dropping_mask_full_rows_cpu_vs_cuda(left):
    """Full rows with either padding side: the device selection agrees with the CPU path (right
    padding's range [1, S) is truncated to the S-1 loss columns, as the reference's slice is)."""
    from centrifuge_b200.loss import token_dropping_mask
    torch.manual_seed(11)
    B, S = 3, 300
    loss = torch.randn(B, S - 1)
    ref = torch.randn(B, S - 1)
    m_cpu = token_dropping_mask(loss, ref, torch.ones(B, S, dtype=torch.long), "fixed", 0.5,
                                left_padding=left)
    m_gpu = token_dropping_mask(loss.to(dev), ref.to(dev),
                                torch.ones(B, S, dtype=torch.long, device=dev), "fixed", 0.5,
                                left_padding=left)
    assert torch.equal(m_gpu.cpu(), m_cpu)


@pytest.mark.parametrize("B,S,nh,nkv,hd", [(2, 256, 4, 2, 64), (1, 200, 4, 1, 128),
                                           (2, 512, 8, 2, 128), (1, 1000, 4, 2, 64),
                                           (1, 2048, 2, 1, 128), (3, 130, 2, 2, 64)])
def test_attention_fwd(B, S, nh, nkv, hd):
    torch.manual_seed(9)
    ld = (nh + 2 * nkv) * hd
    qkv = torch.randn(B * S, ld, device=dev).bfloat16()
    o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd)
    q = qkv[:, : nh * hd].reshape(B, S, nh, hd)
    k = qkv[:, nh * hd:(nh + nkv) * hd].reshape(B, S, nkv, hd)
    v = qkv[:, (nh + nkv) * hd:].reshape(B, S, nkv, hd)
    orf, lr = ref.attention(q, k, v)
    assert rel_err(o, orf.reshape(B * S, nh * hd)) < 1e-2
    assert rel_err(lse, lr.reshape(B * S, nh)) < 1e-4
    from centrifuge_b200.ops import kernels
    assert kernels().gemm_error_word(0, True) == 0
    # the warp-level mma.sync forward agrees too
    o2, l2 = torch.empty_like(o), torch.empty_like(lse)
    kernels().attn_fwd_mma(qkv, o2, l2, B, S, nh, nkv, hd, 1.0 / hd ** 0.5)
    assert rel_err(o2, o) < 1e-2 and rel_err(l2, lse) < 1e-4


@pytest.mark.parametrize("M,F,K", [(4096, 5632, 2048), (1000, 256, 512), (333, 1792, 4096)])
def test_gemm_swiglu_epilogue(M, F, K):
    """Gate/up projection with SwiGLU in the epilogue vs the projection + SwiGLU pass."""
    torch.manual_seed(14)
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(2 * F, K, device=dev) / K ** 0.5).bfloat16()
    gu, h = gemm.linear_fwd_swiglu(x, w)
    y = x.float() @ w.float().t()
    assert rel_err(gu, y) < 1e-2
    assert rel_err(h, ref.swiglu(y)) < 2e-2
    h2 = fused.swiglu_fwd(gu)
    assert (h.float() - h2.float()).abs().max().item() < 2e-2 * max(1.0, h2.float().abs().max().item())


@pytest.mark.parametrize("M,nh,nkv,hd,bn", [(4096, 32, 4, 64, 0), (1000, 8, 2, 128, 128),
                                            (333, 4, 4, 64, 256), (2048, 16, 8, 128, 256),
                                            (1000, 8, 2, 128, 512), (2048, 16, 8, 64, 512)])
def test_gemm_rope_epilogue(M, nh, nkv, hd, bn):
    """QKV projection with RoPE in the epilogue vs the fp32 projection followed by RoPE."""
    from centrifuge_b200.ops import kernels
    torch.manual_seed(12)
    K = 512
    N = (nh + 2 * nkv) * hd
    x = torch.randn(M, K, device=dev).bfloat16()
    w = (torch.randn(N, K, device=dev) / K ** 0.5).bfloat16()
    table = ref.rope_table(4096, hd, 10000.0, dev)
    pos = torch.randint(0, 4096, (M,), device=dev, dtype=torch.int32)
    out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
    kernels().gemm_rope(x, w, out, pos, table, (nh + nkv) * hd, hd, bn)
    y = x.float() @ w.float().t()
    rc = (nh + nkv) * hd
    y[:, :rc] = ref.rope(y[:, :rc].view(M, nh + nkv, hd), pos, table).reshape(M, rc)
    assert rel_err(out, y) < 1e-2
    assert (out.float() - y).abs().max().item() < 0.05
    assert kernels().gemm_error_word(0, True) == 0


@pytest.mark.parametrize("B,S,nh,nkv,hd", [(2, 512, 8, 2, 64), (1, 700, 4, 1, 128)])
def test_attention_bwd_rope_epilogue(B, S, nh, nkv, hd):
    """The RoPE backward folded into the attention backward epilogue equals a separate inverse
    rotation of the dq/dk blocks."""
    torch.manual_seed(13)
    ld = (nh + 2 * nkv) * hd
    qkv = (0.5 * torch.randn(B * S, ld, device=dev)).bfloat16()
    o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd)
    Sk = S // 2
    pos = torch.stack([torch.cat([torch.randperm(S - 1, device=dev)[: Sk - 1].sort().values,
                                  torch.tensor([S - 1], device=dev)]) for _ in range(B)])
    pos = pos.sort(dim=1).values.int()
    flat = (pos + torch.arange(B, device=dev, dtype=torch.int32).view(B, 1) * S).reshape(-1)
    qkv_k, o_k, lse_k = qkv[flat.long()].contiguous(), o[flat.long()].contiguous(), lse[flat.long()].contiguous()
    do_k = torch.randn(B * Sk, nh * hd, device=dev).bfloat16()
    table = ref.rope_table(4096, hd, 500000.0, dev)
    d0 = fused.attn_bwd(qkv_k, qkv, o_k, do_k, lse_k, pos, B, S, Sk, nh, nkv, hd)
    d1 = fused.attn_bwd(qkv_k, qkv, o_k, do_k, lse_k, pos, B, S, Sk, nh, nkv, hd,
                        rope_table=table)
    want = d0.float().clone()
    rc = (nh + nkv) * hd
    want[:, :rc] = ref.rope(want[:, :rc].view(-1, nh + nkv, hd), pos.reshape(-1), table,
                            inverse=True).reshape(-1, rc)
    assert rel_err(d1, want) < 1e-2
    assert torch.equal(d1[:, rc:], d0[:, rc:])


@pytest.mark.parametrize("B,S,nh,nkv,hd,amp", [(8, 2048, 32, 4, 64, 1.0), (4, 2048, 32, 8, 128, 1.0),
                                               (8, 1024, 32, 4, 64, 4.0)])
def test_attention_fwd_many_items(B, S, nh, nkv, hd, amp):
    """More work items than SMs: the persistent kernel runs several items per CTA.  Compared
    element-wise against the warp-level mma.sync forward."""
    from centrifuge_b200.ops import kernels
    torch.manual_seed(11)
    ld = (nh + 2 * nkv) * hd
    qkv = (amp * torch.randn(B * S, ld, device=dev)).bfloat16()
    o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd)
    o2, l2 = torch.empty_like(o), torch.empty_like(lse)
    kernels().attn_fwd_mma(qkv, o2, l2, B, S, nh, nkv, hd, 1.0 / hd ** 0.5)
    assert kernels().gemm_error_word(0, True) == 0
    assert (lse - l2).abs().max().item() < 1e-3
    # against the fp32 oracle, the tcgen05 kernel is as accurate as the mma.sync one
    q = qkv[:, : nh * hd].reshape(B, S, nh, hd)
    k = qkv[:, nh * hd:(nh + nkv) * hd].reshape(B, S, nkv, hd)
    v = qkv[:, (nh + nkv) * hd:].reshape(B, S, nkv, hd)
    orf, _ = ref.attention(q, k, v)
    orf = orf.reshape(B * S, nh * hd)
    e_tc = (o.float() - orf).abs().max().item()
    e_mma = (o2.float() - orf).abs().max().item()
    assert e_tc <= 1.5 * e_mma + 1e-2, (e_tc, e_mma)


@pytest.mark.parametrize("B,S,nh,nkv,hd,keep", [(2, 256, 4, 2, 64, 0.5), (1, 320, 4, 1, 128, 0.3),
                                                (2, 256, 8, 2, 128, 1.0), (1, 128, 2, 2, 64, 0.7),
                                                (2, 1024, 8, 2, 128, 0.5), (1, 700, 4, 4, 64, 0.6),
                                                (2, 2048, 4, 1, 64, 0.5), (1, 96, 2, 1, 128, 0.9)])
def test_attention_bwd_filtered(B, S, nh, nkv, hd, keep):
    torch.manual_seed(10)
    ld = (nh + 2 * nkv) * hd
    qkv = (0.5 * torch.randn(B * S, ld, device=dev)).bfloat16()
    o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd)
    Sk = max(1, int(round(S * keep)))
    pos = torch.stack([torch.cat([torch.randperm(S - 1, device=dev)[: Sk - 1].sort().values,
                                  torch.tensor([S - 1], device=dev)]) for _ in range(B)])
    pos = pos.sort(dim=1).values.int()
    flat = (pos + torch.arange(B, device=dev, dtype=torch.int32).view(B, 1) * S).reshape(-1)
    qkv_k = qkv[flat.long()].contiguous()
    o_k = o[flat.long()].contiguous()
    lse_k = lse[flat.long()].contiguous()
    do_k = torch.randn(B * Sk, nh * hd, device=dev).bfloat16()
    d = fused.attn_bwd(qkv_k, qkv, o_k, do_k, lse_k, pos, B, S, Sk, nh, nkv, hd)
    q = qkv_k[:, : nh * hd].reshape(B, Sk, nh, hd)
    kf = qkv[:, nh * hd:(nh + nkv) * hd].reshape(B, S, nkv, hd)
    vf = qkv[:, (nh + nkv) * hd:].reshape(B, S, nkv, hd)
    dq, dk, dv = ref.attention_bwd_filtered(q, kf, vf, o_k.reshape(B, Sk, nh, hd),
                                            do_k.reshape(B, Sk, nh, hd), lse_k.reshape(B, Sk, nh),
                                            pos)
    assert rel_err(d[:, : nh * hd], dq.reshape(B * Sk, -1)) < 2e-2
    assert rel_err(d[:, nh * hd:(nh + nkv) * hd], dk.reshape(B * Sk, -1)) < 2e-2
    assert rel_err(d[:, (nh + nkv) * hd:], dv.reshape(B * Sk, -1)) < 2e-2
    from centrifuge_b200.ops import kernels
    assert kernels().gemm_error_word(0, True) == 0
    # the warp-level mma.sync backward agrees too
    d2 = torch.empty_like(d)
    delta = torch.empty(B * Sk * nh, dtype=torch.float32, device=dev)
    kernels().attn_bwd_mma(qkv_k, qkv, o_k, do_k, lse_k, pos.reshape(-1), d2, delta, B, S, Sk, nh,
                           nkv, hd, 1.0 / hd ** 0.5)
    assert rel_err(d2, d) < 2e-2


@pytest.mark.parametrize("M,N,K", [(300, 1056, 256), (512, 32000, 2048), (1, 320, 64)])
def test_fused_lm_head_cross_entropy(M, N, K):
    """lm_head GEMM with the cross-entropy statistics in its epilogue (logits never stored) and
    the backward recompute with the dlogits epilogue, against fp32 cross entropy."""
    torch.manual_seed(12)
    x = (torch.randn(M, K, device=dev) * 0.5).bfloat16()
    w = (torch.randn(N, K, device=dev) / K ** 0.5).bfloat16()
    labels = torch.randint(0, N, (M,), device=dev)
    labels[::7] = -100
    loss, lse = gemm.linear_fwd_ce(x, w, labels)
    logits = x.float() @ w.float().t()
    loss_r, lse_r = ref.cross_entropy(logits, labels)
    assert (lse - lse_r).abs().max().item() < 2e-3 * max(1.0, lse_r.abs().max().item())
    assert (loss - loss_r).abs().max().item() < 2e-3 * max(1.0, loss_r.abs().max().item())
    assert bool((loss[labels < 0] == 0).all())
    dloss = torch.rand(M, device=dev)
    g = gemm.linear_ce_grad(x, w, labels, lse, dloss)
    g_r = ref.cross_entropy_bwd(logits, labels, lse_r, dloss)
    err = ((g.float() - g_r).norm() / (g_r.norm() + 1e-12)).item()
    assert err < 1e-2, err
    assert float(g[labels < 0].float().abs().sum()) == 0.0
    from centrifuge_b200.ops import kernels
    assert kernels().gemm_error_word(0, True) == 0
