"""Per-op timing of the tensor-parallel collectives, fused (NVLink / NVSwitch kernels of
``parallel/tp_fused.py``) versus the NCCL baseline, at Llama-3-8B layer shapes.

    torchrun --nproc-per-node P -m centrifuge_b200.benchmarks.tp_comm_bench [--tokens 16384]

Ops (sequence-parallel, T tokens, hidden H, P ranks; fused = one gemm_tp launch after a local
RMSNorm, baseline = RMSNorm + NCCL all-gather + GEMM, or GEMM + NCCL reduce-scatter + add):
  ag_qkv   RMSNorm(local rows) -> all-gather -> QKV projection with RoPE   [T, H] x [H, (nh+2nkv)hd/P]
  ag_gu    RMSNorm -> all-gather -> gate/up projection                       [T, H] x [H, 2F/P]
  rs_o     o projection -> reduce-scatter -> + residual                      [T, nh hd/P] x [., H]
  rs_down  down projection -> reduce-scatter -> + residual                   [T, F/P] x [., H]
Device time with CUDA events over `--iters` launches after warm-up, max over ranks.  The roofline
of an op is the slower of its GEMM at the measured bf16 peak and the bytes that must cross
NVLink per rank ((P-1)/P of the gathered / reduced activation) at 770 GB/s per direction.
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.distributed as dist

PEAK_TFLOPS = 1621.4  # measured cuBLAS bf16 (burst)
LINK_GBS = 770.0      # measured peer copy, per direction


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    from centrifuge_b200.ops import fused
    from centrifuge_b200.ops import gemm as G
    from centrifuge_b200.ops.reference import rope_table
    from centrifuge_b200.parallel.tensor_parallel import TPGroup
    from centrifuge_b200.parallel.tp_fused import TPFusedComm

    P = world
    T, H, nh, nkv, hd, F = a.tokens, 4096, 32, 8, 128, 14336
    tp = TPGroup(dist.group.WORLD)
    comm = TPFusedComm(tp, T, H, 4, dev)
    comm_p2p = TPFusedComm(tp, T, H, 4, dev, use_multicast=False)
    shard = T // P
    g = torch.Generator(device=dev).manual_seed(rank)
    bf = torch.bfloat16

    def rnd(*shape, s=1.0):
        return (s * torch.randn(*shape, generator=g, device=dev)).to(bf)

    x = rnd(shard, H)
    ln = (1 + 0.1 * torch.randn(H, generator=g, device=dev)).to(bf)
    wqkv = rnd((nh + 2 * nkv) * hd // P, H, s=0.02)
    wgu = rnd(2 * F // P, H, s=0.02)
    wo = rnd(H, nh * hd // P, s=0.02)
    wd = rnd(H, F // P, s=0.02)
    o = rnd(T, nh * hd // P)
    h = rnd(T, F // P)
    pos = torch.arange(T, device=dev, dtype=torch.int32) % 4096
    table = rope_table(4096, hd, 500000.0, dev)
    rc = (nh + nkv) * hd // P

    def nccl_ag(w, rope):
        xn, _ = fused.rmsnorm_fwd(x, ln, 1e-5)
        xg = tp.all_gather_rows(xn)
        if rope:
            return G.linear_fwd_rope(xg, w, pos, table, rc, hd)
        return G.linear_fwd(xg, w)

    def fused_ag(w, rope, slot, c=comm):
        xg, _ = c.rmsnorm_local(x, ln, 1e-5, slot)
        return c.gemm_ag(xg, w, slot, rope=(pos, table, rc, hd) if rope else None)

    def nccl_rs(a_, w):
        return tp.reduce_scatter_rows(G.linear_fwd(a_, w)) + x

    def fused_rs(a_, w, c=comm):
        return c.gemm_rs(a_, w, x)

    cp = comm_p2p
    ops = {
        "ag_qkv": (lambda: nccl_ag(wqkv, True), lambda: fused_ag(wqkv, True, 0),
                   lambda: fused_ag(wqkv, True, 0, cp),
                   2.0 * T * H * wqkv.shape[0], (P - 1) / P * T * H * 2),
        "ag_gu": (lambda: nccl_ag(wgu, False), lambda: fused_ag(wgu, False, 1),
                  lambda: fused_ag(wgu, False, 1, cp),
                  2.0 * T * H * wgu.shape[0], (P - 1) / P * T * H * 2),
        "rs_o": (lambda: nccl_rs(o, wo), lambda: fused_rs(o, wo), lambda: fused_rs(o, wo, cp),
                 2.0 * T * wo.shape[1] * H, (P - 1) / P * T * H * 2),
        "rs_down": (lambda: nccl_rs(h, wd), lambda: fused_rs(h, wd), lambda: fused_rs(h, wd, cp),
                    2.0 * T * wd.shape[1] * H, (P - 1) / P * T * H * 2),
    }
    # correctness spot check of the fused ops against NCCL
    for name, (fn_n, fn_f, fn_p, _, _) in ops.items():
        ref = fn_n()
        for tag, fn in (("multicast", fn_f), ("p2p", fn_p)):
            got = fn()
            err = float((got.float() - ref.float()).norm() / (ref.float().norm() + 1e-12))
            if err > 2e-2 and rank == 0:
                print(f"warning: {name} fused ({tag}) vs nccl rel err {err:.3g}", flush=True)

    def time_it(fn):
        for _ in range(a.warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    res = {}
    for name, (fn_n, fn_f, fn_p, flops, link_bytes) in ops.items():
        tn, tf, tp2 = time_it(fn_n), time_it(fn_f), time_it(fn_p)
        roof_ms = max(flops / (PEAK_TFLOPS * 1e12), link_bytes / (LINK_GBS * 1e9)) * 1e3
        res[name] = dict(nccl_ms=tn, fused_multicast_ms=tf, fused_p2p_ms=tp2,
                         roofline_ms=roof_ms, fused_of_roofline=roof_ms / min(tf, tp2),
                         nccl_of_roofline=roof_ms / tn, gemm_tflop=flops / 1e12,
                         link_mb=link_bytes / 1e6)
    if rank == 0:
        print(json.dumps({"P": P, "tokens": T, "comm": comm.kind, "ops": res}, indent=1),
              flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
