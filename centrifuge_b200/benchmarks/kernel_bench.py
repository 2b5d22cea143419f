"""Kernel microbenchmarks: tcgen05 GEMM vs cuBLAS, attention fwd / filtered bwd vs the
reference's ATen attention path (flash + memory-efficient backward) and cuDNN.

    python -m centrifuge_b200.benchmarks.kernel_bench [--json out.json]

Times with CUDA events after warm-up; inputs larger than L2 for the GEMM shapes.
"""
from __future__ import annotations

import argparse
import json
import math

import torch

from centrifuge_b200.ops import fused, gemm


ITERS, WARMUP = 20, 5
LAST_SM_MHZ = [None]


def _sm_mhz():
    """SM clock of device 0 now (NVML), or None."""
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(torch.cuda.current_device())
        return pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
    except Exception:  # pragma: no cover - NVML missing
        return None


def _time(fn, iters=None, warmup=None):
    iters = ITERS if iters is None else iters
    warmup = WARMUP if warmup is None else warmup
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    LAST_SM_MHZ[0] = _sm_mhz()  # read while the queued launches still run
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def bench_gemm(shapes, bn=0, cublas=True, compare=False):
    rows = []
    for (M, N, K, a_mn, b_mn, name) in shapes:
        A = torch.randn(K, M, device="cuda").bfloat16() if a_mn else torch.randn(M, K, device="cuda").bfloat16()
        B = torch.randn(K, N, device="cuda").bfloat16() if b_mn else torch.randn(N, K, device="cuda").bfloat16()
        if a_mn and b_mn:
            # weight gradient: fp32 accumulation into the gradient buffer (split-K when the
            # tile count leaves the last wave mostly empty)
            out = torch.zeros(M, N, device="cuda", dtype=torch.float32)
            epi = gemm.EPI_F32_ACC
        else:
            out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
            epi = gemm.EPI_BF16
        ms = _time(lambda: gemm.gemm(A, B, out, a_mn, b_mn, epi, bn=bn))
        mhz = LAST_SM_MHZ[0]
        # the other tile shapes, timed back to back with the chosen one (same clock regime)
        alt = {}
        for bn_alt in (128, 256, 512):
            if bn_alt != bn and compare:
                t = _time(lambda: gemm.gemm(A, B, out, a_mn, b_mn, epi, bn=bn_alt))
                alt[f"tflops_bn{bn_alt}"] = 2.0 * M * N * K / t / 1e9
        Am = A.t() if a_mn else A
        Bm = B if b_mn else B.t()
        ms_ref = _time(lambda: torch.matmul(Am, Bm)) if cublas else float("nan")
        fl = 2.0 * M * N * K
        rows.append({"name": name, "M": M, "N": N, "K": K, "a_mn": a_mn, "b_mn": b_mn,
                     "ms": ms, "tflops": fl / ms / 1e9, "sm_mhz": mhz, "cublas_ms": ms_ref,
                     "cublas_tflops": fl / ms_ref / 1e9, **alt})
        print(json.dumps(rows[-1]))
    return rows


def bench_fusions(T=16384, Tk=8192, H=2048, F=5632):
    """GEMMs with fused epilogues against the same GEMM followed by the separate kernel, at the
    TinyLlama MLP shapes (T tokens forward, Tk kept rows backward); times back to back."""
    from centrifuge_b200.ops import fused
    x = torch.randn(T, H, device="cuda").bfloat16()
    wgu = (torch.randn(2 * F, H, device="cuda") / H ** 0.5).bfloat16()
    wd = (torch.randn(H, F, device="cuda") / F ** 0.5).bfloat16()
    dy = torch.randn(Tk, H, device="cuda").bfloat16()
    rows = torch.randperm(T, device="cuda")[:Tk].sort().values.int()
    gu, _ = gemm.linear_fwd_swiglu(x, wgu)
    res = []

    def unfused_fwd():
        g = gemm.linear_fwd(x, wgu)
        return fused.swiglu_fwd(g)

    def unfused_bwd():
        dh = gemm.linear_dgrad(dy, wd)
        return fused.swiglu_bwd(dh, gu, rows)

    for name, f_fused, f_sep, fl in (
            ("swiglu_fwd_gemm", lambda: gemm.linear_fwd_swiglu(x, wgu), unfused_fwd,
             2.0 * T * H * 2 * F),
            ("swiglu_bwd_gemm", lambda: gemm.linear_dgrad_swiglu(dy, wd, gu, rows), unfused_bwd,
             2.0 * Tk * H * F)):
        t_f = _time(f_fused)
        t_s = _time(f_sep)
        res.append({"name": name, "fused_ms": t_f, "separate_ms": t_s,
                    "fused_tflops": fl / t_f / 1e9, "separate_tflops": fl / t_s / 1e9})
        print(json.dumps(res[-1]))
    return res


def _heads_major(x, B, S, n, hd):
    """[B*S, n*hd] token-major rows -> [B, n, S, hd] (a view)."""
    return x.view(B, S, n, hd).transpose(1, 2)


def _repeat_kv(x, rep):
    """[B, nkv, S, hd] -> [B, nkv*rep, S, hd] (K/V repeated per query head, as the reference's
    pinned transformers does before SDPA)."""
    B, n, S, hd = x.shape
    return x[:, :, None].expand(B, n, rep, S, hd).reshape(B, n * rep, S, hd)


def bench_attention_reference(qkv, B, S, nh, nkv, hd, pos_by_keep, res):
    """The reference's attention on ATen kernels, same shapes.

    Forward: dense causal flash attention over K/V repeated to the query heads (HF SDPA path of
    transformers 4.45.2).  Filtered backward (grad_filter/token_filter/csrc/backward_filters.cpp:
    420-486, RESTORE_Q): flash attention backward over kept queries x kept keys (is_causal), plus
    the memory-efficient attention backward over kept queries x dropped keys with a
    [B, heads, S_keep, S_drop] additive causal bias, whose dQ is added to the first; dK/dV of
    the dropped keys are computed there and discarded, as in the reference.  The bias is built
    once outside the timed region (the reference builds it once per graph).  Also timed: the
    dense flash backward and cuDNN attention forward + backward (unfiltered baselines).
    """
    aten = torch.ops.aten
    scale = 1.0 / math.sqrt(hd)
    rep = nh // nkv
    q = _heads_major(qkv[:, :nh * hd], B, S, nh, hd)
    k = _repeat_kv(_heads_major(qkv[:, nh * hd:(nh + nkv) * hd], B, S, nkv, hd), rep)
    v = _repeat_kv(_heads_major(qkv[:, (nh + nkv) * hd:], B, S, nkv, hd), rep)
    fwd = aten._scaled_dot_product_flash_attention(q, k, v, 0.0, True, False, scale=scale)
    out, lse, cq, ck, mq, mk, seed, off = fwd[:8]
    fl_f = 4.0 * B * nh * hd * S * S / 2
    ms = _time(lambda: aten._scaled_dot_product_flash_attention(q, k, v, 0.0, True, False,
                                                                scale=scale), iters=10)
    res.append({"name": "aten_flash_fwd_dense", "ms": ms, "tflops": fl_f / ms / 1e9})
    print(json.dumps(res[-1]))
    dout = torch.randn_like(out)
    ms = _time(lambda: aten._scaled_dot_product_flash_attention_backward(
        dout, q, k, v, out, lse, cq, ck, mq, mk, 0.0, True, seed, off, scale=scale), iters=10)
    res.append({"name": "aten_flash_bwd_dense", "ms": ms, "tflops": 2.5 * fl_f / ms / 1e9})
    print(json.dumps(res[-1]))
    try:
        qc = q.detach().clone().requires_grad_()
        kc = _heads_major(qkv[:, nh * hd:(nh + nkv) * hd], B, S, nkv, hd).detach().clone()
        vc = _heads_major(qkv[:, (nh + nkv) * hd:], B, S, nkv, hd).detach().clone()
        kc.requires_grad_()
        vc.requires_grad_()
        from torch.nn.attention import SDPBackend, sdpa_kernel
        with sdpa_kernel(SDPBackend.CUDNN_ATTENTION):
            o_c = torch.nn.functional.scaled_dot_product_attention(qc, kc, vc, is_causal=True,
                                                                   enable_gqa=True)
            ms_f = _time(lambda: torch.nn.functional.scaled_dot_product_attention(
                qc, kc, vc, is_causal=True, enable_gqa=True), iters=10)
            g_c = torch.randn_like(o_c)

            def fb():
                o2 = torch.nn.functional.scaled_dot_product_attention(qc, kc, vc, is_causal=True,
                                                                      enable_gqa=True)
                torch.autograd.grad(o2, (qc, kc, vc), g_c)

            ms_fb = _time(fb, iters=10)
        res.append({"name": "cudnn_fwd_dense", "ms": ms_f, "tflops": fl_f / ms_f / 1e9})
        print(json.dumps(res[-1]))
        res.append({"name": "cudnn_bwd_dense", "ms": ms_fb - ms_f,
                    "tflops": 2.5 * fl_f / (ms_fb - ms_f) / 1e9})
        print(json.dumps(res[-1]))
    except Exception as e:  # cuDNN attention unavailable for this shape
        res.append({"name": "cudnn_dense", "error": str(e)[:200]})
        print(json.dumps(res[-1]))
    for keep, pos in pos_by_keep:
        Sk = pos.shape[1]
        Sd = S - Sk
        keepm = torch.zeros(B, S, dtype=torch.bool, device="cuda")
        keepm.scatter_(1, pos.long(), True)
        drop = torch.stack([torch.nonzero(~keepm[b]).squeeze(1) for b in range(B)])

        def rows(t, idx):  # [B, h, S, hd] -> [B, h, len(idx), hd] per batch row
            return torch.stack([t[b].index_select(1, idx[b]) for b in range(B)]).contiguous()

        q_k, k_k, v_k = rows(q, pos.long()), rows(k, pos.long()), rows(v, pos.long())
        o_k = rows(out, pos.long())
        lse_k = torch.stack([lse[b].index_select(1, pos[b].long()) for b in range(B)]).contiguous()
        do_k = torch.randn_like(o_k)
        fl = 4.0 * B * nh * hd * (Sk * Sk / 2) + 6.0 * B * nh * hd * (Sk * S / 2)
        if Sd > 0:
            k_d, v_d = rows(k, drop), rows(v, drop)
            causal = torch.full((S, S), float("-inf"), device="cuda").triu_(1)
            bias = torch.stack([causal.index_select(0, pos[b].long()).index_select(1, drop[b])
                                for b in range(B)]).to(q.dtype)
            bias = bias[:, None].expand(B, nh, Sk, Sd).contiguous()
            zero = torch.zeros(1, dtype=torch.long, device="cuda")

        def ref_bwd():
            dq, dk, dv = aten._scaled_dot_product_flash_attention_backward(
                do_k, q_k, k_k, v_k, o_k, lse_k, cq, ck, Sk, Sk, 0.0, True, seed, off,
                scale=scale)
            if Sd > 0:
                r = aten._scaled_dot_product_efficient_attention_backward(
                    do_k, q_k, k_d, v_d, bias, o_k, lse_k, zero, zero, 0.0,
                    [True, True, True, False], False, scale=scale)
                dq.add_(r[0])
            return dq

        try:
            ms = _time(ref_bwd, iters=10)
            res.append({"name": f"reference_aten_bwd_keep{keep}", "Sk": Sk, "ms": ms,
                        "tflops": fl / ms / 1e9})
        except Exception as e:
            res.append({"name": f"reference_aten_bwd_keep{keep}", "Sk": Sk,
                        "error": str(e)[:300]})
        print(json.dumps(res[-1]))


def bench_attention(B=4, S=4096, nh=32, nkv=8, hd=128, keeps=(1.0, 0.7, 0.5, 0.3),
                    reference=True):
    ld = (nh + 2 * nkv) * hd
    qkv = torch.randn(B * S, ld, device="cuda").bfloat16()
    o, lse = fused.attn_fwd(qkv, B, S, nh, nkv, hd)
    ms_f = _time(lambda: fused.attn_fwd(qkv, B, S, nh, nkv, hd, out=o, lse=lse), iters=10)
    fl_f = 4.0 * B * nh * hd * S * S / 2
    res = [{"name": "attn_fwd_tcgen05", "ms": ms_f, "tflops": fl_f / ms_f / 1e9}]
    print(json.dumps(res[-1]))
    from centrifuge_b200.ops import kernels
    ms_m = _time(lambda: kernels().attn_fwd_mma(qkv, o, lse, B, S, nh, nkv, hd, 1.0 / hd ** 0.5),
                 iters=10)
    res.append({"name": "attn_fwd_mma_sync", "ms": ms_m, "tflops": fl_f / ms_m / 1e9})
    print(json.dumps(res[-1]))
    if hd == 128:
        q64 = torch.randn(B * S, (nh + 2 * nkv) * 64, device="cuda").bfloat16()
        o64, l64 = fused.attn_fwd(q64, B, S, nh, nkv, 64)
        ms64 = _time(lambda: fused.attn_fwd(q64, B, S, nh, nkv, 64, out=o64, lse=l64), iters=10)
        res.append({"name": "attn_fwd_tcgen05_hd64", "ms": ms64,
                    "tflops": fl_f / 2 / ms64 / 1e9})
        print(json.dumps(res[-1]))
    g = torch.Generator(device="cuda").manual_seed(0)
    pos_by_keep = []
    for keep in keeps:
        Sk = int(S * keep) // 8 * 8
        pos = torch.stack([torch.randperm(S, device="cuda", generator=g)[:Sk].sort().values
                           for _ in range(B)]).int()
        pos_by_keep.append((keep, pos))
        flat = (pos + torch.arange(B, device="cuda", dtype=torch.int32).view(B, 1) * S).reshape(-1)
        qkv_k = qkv[flat.long()].contiguous()
        o_k = o[flat.long()].contiguous()
        lse_k = lse[flat.long()].contiguous()
        do_k = torch.randn(B * Sk, nh * hd, device="cuda").bfloat16()
        dq = torch.empty_like(qkv_k)
        ms = _time(lambda: fused.attn_bwd(qkv_k, qkv, o_k, do_k, lse_k, pos, B, S, Sk, nh, nkv, hd,
                                          dqkv_k=dq), iters=10)
        # useful flops: dK/dV part over kept x kept (causal) + dQ part over kept x all keys
        fl = 4.0 * B * nh * hd * (Sk * Sk / 2) + 6.0 * B * nh * hd * (Sk * S / 2)
        res.append({"name": f"attn_bwd_keep{keep}", "Sk": Sk, "ms": ms, "tflops": fl / ms / 1e9})
        print(json.dumps(res[-1]))
        if keep == keeps[0]:
            delta = torch.empty(B * Sk * nh, dtype=torch.float32, device="cuda")
            ms_m = _time(lambda: kernels().attn_bwd_mma(qkv_k, qkv, o_k, do_k, lse_k,
                                                        pos.reshape(-1), dq, delta, B, S, Sk, nh,
                                                        nkv, hd, 1.0 / hd ** 0.5), iters=10)
            res.append({"name": f"attn_bwd_mma_sync_keep{keep}", "Sk": Sk, "ms": ms_m,
                        "tflops": fl / ms_m / 1e9})
            print(json.dumps(res[-1]))
    if reference:
        bench_attention_reference(qkv, B, S, nh, nkv, hd, pos_by_keep, res)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--skip-attn", action="store_true")
    ap.add_argument("--skip-gemm", action="store_true")
    ap.add_argument("--fusions", action="store_true",
                    help="fused-epilogue GEMMs vs GEMM + separate kernel (MLP shapes)")
    ap.add_argument("--attn-shape", default="4,4096,32,8,128",
                    help="B,S,nh,nkv,hd of the attention benchmark")
    ap.add_argument("--shapes", default=None, help="comma-separated GEMM shape names")
    ap.add_argument("--bn", type=int, default=0, help="GEMM tile width (128, 256; 0 = auto)")
    ap.add_argument("--no-cublas", action="store_true")
    ap.add_argument("--compare-tiles", action="store_true",
                    help="also time every fixed tile shape (bn 128, 256, 512 = CTA pair)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--no-reference", action="store_true",
                    help="skip the reference's ATen attention path (flash + efficient bwd)")
    ap.add_argument("--keeps", default="1.0,0.7,0.5,0.3",
                    help="kept fractions of the filtered attention backward benchmark")
    args = ap.parse_args()
    shapes = [
        (8192, 8192, 8192, False, False, "square"),
        (16384, 2560, 2048, False, False, "tinyllama_qkv_fwd"),
        (16384, 11264, 2048, False, False, "tinyllama_gateup_fwd"),
        (16384, 2048, 5632, False, False, "tinyllama_down_fwd"),
        (8192, 2048, 5632, False, True, "tinyllama_down_dgrad_kept"),
        (2048, 5632, 8192, True, True, "tinyllama_down_wgrad_kept"),
        (2560, 2048, 8192, True, True, "tinyllama_qkv_wgrad_kept"),
        (2048, 2048, 8192, True, True, "tinyllama_o_wgrad_kept"),
        (11264, 2048, 8192, True, True, "tinyllama_gateup_wgrad_kept"),
        (16384, 32000, 2048, False, False, "tinyllama_lmhead_fwd"),
    ]
    global ITERS, WARMUP
    ITERS, WARMUP = args.iters, args.warmup
    if args.shapes:
        keep = set(args.shapes.split(","))
        shapes = [sh for sh in shapes if sh[-1] in keep]
    out = {}
    if not args.skip_gemm:
        out["gemm"] = bench_gemm(shapes, bn=args.bn, cublas=not args.no_cublas,
                                 compare=args.compare_tiles)
    if args.fusions:
        out["fusions"] = bench_fusions()
    if not args.skip_attn:
        B, S, nh, nkv, hd = (int(x) for x in args.attn_shape.split(","))
        keeps = tuple(float(x) for x in args.keeps.split(","))
        out["attention"] = bench_attention(B, S, nh, nkv, hd, keeps=keeps,
                                           reference=not args.no_reference)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
