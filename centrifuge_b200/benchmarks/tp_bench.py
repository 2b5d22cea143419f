"""Tensor / pipeline parallel benchmark (Llama-3-8B workloads).

    torchrun --nproc-per-node 8 -m centrifuge_b200.benchmarks.tp_bench --tp 8 --drop 0.5
    torchrun --nproc-per-node 8 -m centrifuge_b200.benchmarks.tp_bench --tp 4 --pp 2 --mbs 2 --micro 8

* TP=8 + sequence parallel: Llama-3-8B, sequence 4096, global batch 32 sequences per step
  (``--mbs`` sequences per micro-batch, ``32 / mbs`` micro-batches), filter ratios 0/30/50/70%.
* TP=4 x PP=2: 1F1B with 8 micro-batches of 2 x 4096 tokens, 50% filtering.
Device-timed with CUDA events (barrier + synchronize around K steps), max over ranks; rank 0
prints one JSON line per run.  Random-init weights, uniform token ids, LogNormal(1, 0.5)
reference loss.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys

import torch
import torch.distributed as dist


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="llama-3-8b")
    ap.add_argument("--layers", type=int, default=None, help="override layer count (smoke runs)")
    ap.add_argument("--tp", type=int, default=8)
    ap.add_argument("--pp", type=int, default=1)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--mbs", type=int, default=4)
    ap.add_argument("--global_batch", type=int, default=32)
    ap.add_argument("--micro", type=int, default=None, help="pipeline micro-batches")
    ap.add_argument("--head-cost", type=float, default=None,
                    help="LM head + loss cost in decoder layers for the stage split (default: "
                         "FLOP estimate; stage busy times at Llama-3-8B TP2 S4096 measured ~5)")
    ap.add_argument("--even-stages", action="store_true",
                    help="split layers evenly over pipeline stages (default: balance the LM "
                         "head's cost)")
    ap.add_argument("--drop", type=float, nargs="+", default=[0.5])
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"],
                    help="fused: collectives fused into RMSNorm / the GEMMs over NVLink "
                         "(tensor-parallel without pipeline stages); nccl: NCCL all-gather / "
                         "reduce-scatter (the baseline)")
    a = ap.parse_args()

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                            device_id=torch.device("cuda", local))
    rank, world = dist.get_rank(), dist.get_world_size()
    assert world == a.tp * a.pp
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
    from centrifuge_b200.config import get_model_config
    from centrifuge_b200.models.tp_llama import TPLlamaCore
    from centrifuge_b200.parallel.pipeline import (PipelineTrainer, build_groups,
                                                   head_cost_layers, stage_layers)
    from centrifuge_b200.parallel.zero import ZeroAdamW
    from centrifuge_b200.trainer import Trainer
    from centrifuge_b200.data.synthetic import SyntheticTokenData

    cfg = get_model_config(a.model)
    if a.layers:
        cfg.num_hidden_layers = a.layers
    cfg.max_position_embeddings = max(cfg.max_position_embeddings, a.seq)
    dev = torch.device("cuda", local)
    g = build_groups(a.tp, a.pp)
    # stages balanced by cost (the last one also runs the LM head) unless --even-stages
    hc = 0.0 if a.even_stages else (a.head_cost if a.head_cost is not None
                                    else head_cost_layers(cfg, a.seq))
    layers = stage_layers(cfg.num_hidden_layers, a.pp, g.stage, head_cost=hc)
    core = TPLlamaCore(cfg, g.tp_group, device=dev, first=layers.start, last=layers.stop,
                       has_embed=g.stage == 0, has_head=g.stage == a.pp - 1)
    core.use_fused_comm = a.comm == "fused" and a.tp > 1
    core.comm_sets = a.pp  # 1F1B keeps up to pp forwarded micro-batches per stage
    gen = torch.Generator(device=dev).manual_seed(1234 + g.stage * 100 + g.tp_rank)
    for name, p in core.flat.params.items():
        if p.dim() == 1:
            p.fill_(1.0)
        else:
            p.normal_(0.0, cfg.initializer_range, generator=gen)
    opt = ZeroAdamW(core.flat, group=None, lr=1e-4, betas=(0.9, 0.95), grad_clip=1.0,
                    norm_group=dist.group.WORLD, replicated_ranges=core.replicated_ranges(),
                    replication=a.tp)
    M = a.micro or max(1, a.global_batch // a.mbs)
    data = SyntheticTokenData(cfg.vocab_size, a.mbs, a.seq, seed=4321)  # same data on all ranks
    for drop in a.drop:
        if a.pp > 1:
            tr = PipelineTrainer(core, opt, g, drop_rate=drop, num_microbatches=M)
            batches = [(b.input_ids.to(dev), b.ref_loss.to(dev)) for b in (data.sample() for _ in range(M))]
            step = lambda: tr.train_step(batches)  # noqa: E731
        else:
            opt.pre_step_hooks = [core.reduce_replicated_grads]
            tr = Trainer(core, opt, drop_rate=drop, grad_accum=M, world_size=1)
            batches = [data.sample().to(dev) for _ in range(M)]
            step = lambda: tr.train_step(batches, to_device=False)  # noqa: E731
        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize()
        if a.pp > 1:
            tr.timing = True
            tr.busy_ms()
        dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.steps):
            step()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t) / a.steps
        tokens = M * a.mbs * a.seq
        pipe = {}
        if a.pp > 1:
            # bubble of this stage = 1 - (its compute time / step time); 1F1B theory for equal
            # stages: (pp - 1) / (M + pp - 1)
            busy = tr.busy_ms() / a.steps
            tr.timing = False
            b = torch.tensor([1.0 - busy / ms, busy], device=dev)
            bmax, bmin = b.clone(), b.clone()
            dist.all_reduce(bmax, op=dist.ReduceOp.MAX)
            dist.all_reduce(bmin, op=dist.ReduceOp.MIN)
            pipe = {"bubble_fraction_max": float(bmax[0]), "bubble_fraction_min": float(bmin[0]),
                    "stage_busy_ms_max": float(bmax[1]), "stage_busy_ms_min": float(bmin[1]),
                    "bubble_1f1b_theory": (a.pp - 1) / (M + a.pp - 1)}
        if rank == 0:
            print(json.dumps({
                "metric": "train tokens/sec (device-timed, max over ranks)",
                "value": tokens / (ms / 1000), "unit": "tokens/s", "n_gpus": world,
                "ms_per_step": ms, "steps": a.steps, "warmup": a.warmup, "drop_rate": drop,
                "config": {"model": cfg.name, "layers": cfg.num_hidden_layers, "seq_len": a.seq,
                           "stage0_layers": len(stage_layers(cfg.num_hidden_layers, a.pp, 0,
                                                             head_cost=hc)),
                           "micro_batch": a.mbs, "micro_batches": M,
                           "global_batch": M * a.mbs,
                           "parallelism": f"tp{a.tp}" + (f"pp{a.pp}-1f1b" if a.pp > 1 else "-sp")},
                "comm": (core._comm.kind if core._comm is not None else "nccl"),
                **({"pipeline": pipe} if pipe else {}),
                "dtype": "bf16", "data": "synthetic"}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
