"""Headline benchmark: filtered training throughput of TinyLlama-1.1B, ZeRO-2 data parallel.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--drop 0.5] [--impl native|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Workload: TinyLlama-1.1B architecture (random init), bf16, sequence 2048, micro-batch 8,
gradient accumulation 4 (per GPU: weak scaling), fused AdamW (lr 1e-4, betas 0.9/0.95),
gradient clip 1.0, ZeRO stage 2, 50% backward token filtering by excess loss over a synthetic
per-token reference loss (uniform token ids, LogNormal(1.0, 0.5) ref_loss).

Two measurements, rank 0 prints one JSON line:
* ``value``: device-timed tokens/s (CUDA events on the launching stream, barrier +
  synchronize around exactly K steps, max over ranks), with each step's inputs already on the
  device.  The working set (2.2 GB of weights, ~20 GB of activations per micro-batch) is far
  larger than the 126 MB L2.
* ``e2e``: the same training step through the public API (``Trainer.train_step``) with every
  step's inputs copied host->device from pinned memory and the loss read back to the host.

``--impl reference`` replaces this process by ``baseline/ref_arm.py``: the reference
implementation's own training step (HF Llama + its ``token_filter_loss`` + its
``backward_filter_with_dims`` extension) on the same workload, built by
``baseline/build_ref.sh`` into ``baseline/_ref``.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import subprocess
import sys
import time

import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from baseline.clocks import ClockSampler  # noqa: E402

METRIC = "train tokens/sec (device-timed, max over ranks) @50% filter at 1/2/4/8 B200 vs ref build"
REF_DIR = os.path.join(ROOT, "baseline", "_ref")
REF_ARM = os.path.join(ROOT, "baseline", "ref_arm.py")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--model", default="tinyllama-1.1b")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--mbs", type=int, default=8)
    ap.add_argument("--ga", type=int, default=4)
    ap.add_argument("--drop", type=float, default=0.5)
    ap.add_argument("--mode", default="centrifuge", choices=["regular", "loss_only", "centrifuge"],
                    help="regular: no filtering; loss_only: filtered loss, dense backward; "
                         "centrifuge: filtered loss and filtered backward")
    ap.add_argument("--zero", type=int, default=2)
    ap.add_argument("--reducer", default="auto", choices=["auto", "nccl", "symm"])
    ap.add_argument("--grad-mode", default="ring", choices=["ring", "full"],
                    help="ring: partitioned ZeRO-2 gradients (bucket slots, reduce-scatter in "
                         "every micro-batch); full: full fp32 local gradients reduced once per "
                         "step (ZeRO-1 gradient memory)")
    ap.add_argument("--layers", type=int, default=None,
                    help="override the layer count (quick checks only; not a benchmark config)")
    ap.add_argument("--no-status", action="store_true",
                    help="do not read the device status word each step (A/B of its cost)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--json-out", default=None)
    return ap.parse_args()


def init_dist(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    return world, rank, local


def _reference_built() -> bool:
    so = os.path.join(REF_DIR, "grad_filter", "token_filter")
    return os.path.isdir(so) and any(f.startswith("_C") and f.endswith(".so") for f in os.listdir(so))


def run_reference(args):
    """Replace this process by the reference arm (baseline/ref_arm.py), which runs the
    reference's own training step; build the reference first if baseline/_ref is missing."""
    rank = int(os.environ.get("RANK", "0"))
    if not _reference_built() and rank == 0:
        subprocess.run(["bash", os.path.join(ROOT, "baseline", "build_ref.sh")], check=False)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # every rank waits for rank 0's build through the filesystem (no process group yet)
        for _ in range(600):
            if _reference_built():
                break
            time.sleep(1)
    if not _reference_built():
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable":
                              "the reference's grad_filter extension is not built and "
                              "baseline/build_ref.sh could not build it here"}), flush=True)
        return
    argv = [sys.executable, REF_ARM] + sys.argv[1:]
    sys.stdout.flush()
    os.execv(sys.executable, argv)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    world, rank, local = init_dist(args)
    if args.gpus != world and rank == 0:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE {world}", file=sys.stderr)
    from centrifuge_b200.config import get_model_config
    from centrifuge_b200.data.synthetic import SyntheticTokenData
    from centrifuge_b200.models.llama import NativeLlamaForCausalLM
    from centrifuge_b200.ops._ext import counter
    from centrifuge_b200.parallel.zero import ZeroAdamW
    from centrifuge_b200.trainer import Trainer

    dev = torch.device("cuda", local)
    cfg = get_model_config(args.model)
    cfg.max_position_embeddings = max(cfg.max_position_embeddings, args.seq)
    if args.layers:
        cfg.num_hidden_layers = args.layers
    model = NativeLlamaForCausalLM(cfg, device=dev, seed=4321, pad_to=world)
    group = dist.group.WORLD if world > 1 else None
    reducer = None
    if world > 1 and args.reducer in ("auto", "symm"):
        try:
            from centrifuge_b200.parallel.symm import SymmReducer
            reducer = SymmReducer.create(model.flat, group, ring=args.grad_mode == "ring")
        except Exception as e:  # the NCCL baseline stays available
            if args.reducer == "symm":
                raise
            if rank == 0:
                print(f"symmetric-memory reducer unavailable ({e}); using NCCL", file=sys.stderr)
    opt = ZeroAdamW(model.flat, group=group, stage=args.zero, lr=1e-4, betas=(0.9, 0.95),
                    eps=1e-8, weight_decay=0.0, grad_clip=1.0, reducer=reducer,
                    grad_mode=args.grad_mode if args.zero == 2 else "full")
    drop = 0.0 if args.mode == "regular" else args.drop
    trainer = Trainer(model, opt, drop_rate=drop, grad_accum=args.ga, world_size=world,
                      filter_backward=args.mode == "centrifuge",
                      check_device_errors=not args.no_status)
    data = SyntheticTokenData(cfg.vocab_size, args.mbs, args.seq, seed=4321, rank=rank)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- device-timed loop: inputs staged on the device
    dev_batches = [data.sample().to(dev) for _ in range(args.ga)]
    for _ in range(args.warmup):
        trainer.train_step(dev_batches, to_device=False)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    counter.reset()
    torch.cuda.reset_peak_memory_stats(dev)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        start.record()
        for _ in range(args.steps):
            loss = trainer.train_step(dev_batches, to_device=False)
        stop.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    launches = counter.reset()
    peak_gb = torch.cuda.max_memory_allocated(dev) / 2 ** 30
    ms = start.elapsed_time(stop)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = world * args.ga * args.mbs * args.seq * args.steps
    value = tokens / (ms_max / 1000.0)

    # ---- end-to-end loop through the public API: H2D per step + loss readout
    e2e = None
    if not args.no_e2e:
        host_batches = [[data.sample() for _ in range(args.ga)] for _ in range(args.steps)]
        h2d = sum(b.nbytes() for b in host_batches[0])
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for step in range(args.steps):
            loss_val = trainer.train_step(host_batches[step], to_device=True).item()
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        tw = torch.tensor([wall], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tw, op=dist.ReduceOp.MAX)
        e2e = {"value": tokens / float(tw.item()), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
               "loss_last": loss_val, "device_ms": e0.elapsed_time(e1)}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform token ids, LogNormal(1.0,0.5) ref_loss, random-init weights)",
            "config": {"model": cfg.name, "global_batch": world * args.ga * args.mbs,
                       "micro_batch": args.mbs, "grad_accum": args.ga, "seq_len": args.seq,
                       "drop_rate": drop, "mode": args.mode,
                       "parallelism": f"zero{args.zero}-dp{world}",
                       "grad_mode": opt.grad_mode,
                       "grad_memory_gib": round(opt.grad_memory_bytes() / 2 ** 30, 3),
                       "layers": cfg.num_hidden_layers,
                       "reducer": (getattr(opt.reducer, "kind", type(opt.reducer).__name__)
                                   if opt.reducer else "none"),
                       "l2": "working set (weights + activations) far larger than L2"},
            "clocks": clocks.summary(), "gpu_launches": launches, "e2e": e2e,
            "peak_mem_gib": round(peak_gb, 2),
            "loss": float(loss.item()),
        }
        print(json.dumps(line), flush=True)
        if args.json_out:
            with open(args.json_out, "w") as f:
                json.dump(line, f, indent=1)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
