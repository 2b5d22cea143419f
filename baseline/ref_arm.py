"""Reference arm of bench.py: the reference implementation's own filtered training step.

    python baseline/ref_arm.py --gpus N --steps K --warmup W [--mode centrifuge|loss_only|regular]
    (bench.py --impl reference execs this file; torchrun launches it the same way for N > 1)

Runs the UNMODIFIED reference (Di-Chai/Centrifuge), built by ``baseline/build_ref.sh`` into
``baseline/_ref``, through its public API and stock code path, on the same workload as the
native arm: TinyLlama-1.1B architecture (random init), bf16, sequence 2048, micro-batch 8,
gradient accumulation 4 per GPU, 50% backward token filtering by excess loss over a synthetic
LogNormal(1.0, 0.5) per-token reference loss, AdamW (lr 1e-4, betas 0.9/0.95), clip 1.0.

Per micro-batch the sequence is the reference's ``Trainer.train_step`` (train.py:222-326):
HF ``LlamaForCausalLM`` forward (SDPA attention, cuBLAS GEMMs), ``model.utils.token_filter_loss``
(``fixed`` strategy, returns the mask), the all-token loss, the filtering-ratio readout,
``token_filter.ops.backward_filter_with_dims`` with the dims recorded once on a probe batch by
``gen_node_tracing.gen_node_tracing_with_model_with_dims`` (bsz 19, seq 224, as train.py:100-103),
the loss readouts, ``backward`` of the loss scaled by 1/grad_accum (what DeepSpeed's
``engine.backward`` does), and the ``torch.cuda.synchronize()`` calls train_step makes.

Stand-ins (declared in the JSON line): DeepSpeed is not installed, so its bf16 ZeRO-1 engine
(train.py:115-175) is replaced by the same algorithm on stock torch + NCCL: bf16 parameters in
one flat buffer, fp32 gradients accumulated after every micro-batch, at the accumulation boundary
an NCCL reduce-scatter of the fp32 gradients, global-norm clipping, ``torch.optim.AdamW
(fused=True)`` on the rank's fp32 master shard and an NCCL all-gather of the bf16 parameters.  The
WarmupCosineLR schedule is left out (constant lr).  Nothing from ``centrifuge_b200`` is imported.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
REF = os.path.join(HERE, "_ref")
# The repository root holds a ``grad_filter`` compatibility package of the new framework; keep
# it off the path so ``from grad_filter import token_filter`` resolves to the reference's build.
sys.path[:] = [p for p in sys.path if os.path.abspath(p or os.getcwd()) != REPO]
sys.path.insert(0, REF)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from clocks import ClockSampler  # noqa: E402  (baseline/clocks.py)

METRIC = "train tokens/sec (device-timed, max over ranks) @50% filter at 1/2/4/8 B200 vs ref build"
TINYLLAMA = dict(hidden_size=2048, intermediate_size=5632, num_hidden_layers=22,
                 num_attention_heads=32, num_key_value_heads=4, vocab_size=32000,
                 rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=2048,
                 tie_word_embeddings=False, hidden_act="silu")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--mbs", type=int, default=8)
    ap.add_argument("--ga", type=int, default=4)
    ap.add_argument("--drop", type=float, default=0.5)
    ap.add_argument("--layers", type=int, default=None, help="override the layer count (tests)")
    ap.add_argument("--mode", default="centrifuge", choices=["regular", "loss_only", "centrifuge"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--json-out", default=None)
    ap.add_argument("--impl", default="reference")  # accepted for bench.py's command line
    ap.add_argument("--model", default="tinyllama-1.1b")
    ap.add_argument("--zero", type=int, default=2)
    ap.add_argument("--reducer", default="nccl")
    args, _ = ap.parse_known_args()
    return args


class ZeroOneBF16:
    """DeepSpeed bf16 ZeRO stage-1 stand-in on stock torch + NCCL (see module docstring)."""

    def __init__(self, model, world, rank, lr, betas, eps, weight_decay, clip):
        params = [p for p in model.parameters() if p.requires_grad]
        self.params = params
        n = sum(p.numel() for p in params)
        self.world, self.rank, self.clip = world, rank, clip
        self.numel = -(-n // world) * world
        dev = params[0].device
        self.flat = torch.zeros(self.numel, dtype=torch.bfloat16, device=dev)
        off = 0
        for p in params:
            k = p.numel()
            self.flat[off:off + k].copy_(p.data.flatten())
            p.data = self.flat[off:off + k].view_as(p)
            off += k
        self.grad32 = torch.zeros(self.numel, dtype=torch.float32, device=dev)
        off, self.gviews = 0, []
        for p in params:
            self.gviews.append(self.grad32[off:off + p.numel()].view_as(p))
            off += p.numel()
        shard = self.numel // world
        self.lo, self.hi = rank * shard, (rank + 1) * shard
        self.master = torch.nn.Parameter(self.flat[self.lo:self.hi].float())
        self.gshard = torch.zeros(shard, dtype=torch.float32, device=dev)
        self.opt = torch.optim.AdamW([self.master], lr=lr, betas=betas, eps=eps,
                                     weight_decay=weight_decay, fused=True)

    def accumulate(self):
        grads = [p.grad for p in self.params]
        torch._foreach_add_(self.gviews, grads)
        for p in self.params:
            p.grad = None

    def step(self):
        if self.world > 1:
            dist.reduce_scatter_tensor(self.gshard, self.grad32, op=dist.ReduceOp.AVG)
        else:
            self.gshard.copy_(self.grad32)
        sq = self.gshard.square().sum()
        if self.world > 1:
            dist.all_reduce(sq)
        coef = torch.clamp(self.clip / (sq.sqrt() + 1e-6), max=1.0)
        self.master.grad = self.gshard.mul_(coef)
        self.opt.step()
        self.master.grad = None
        if self.world > 1:
            dist.all_gather_into_tensor(self.flat, self.master.detach().to(torch.bfloat16))
        else:
            self.flat.copy_(self.master.detach())
        self.grad32.zero_()


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)

    from transformers import LlamaConfig, LlamaForCausalLM
    from transformers.integrations import sdpa_attention

    # The reference pins transformers 4.45.2 (docker/Dockerfile:26), whose Llama attention
    # repeats K/V to the query head count before SDPA.  transformers 5.5 instead passes
    # enable_gqa=True with 4 K/V heads, which the reference's restore-Q attention node does not
    # handle (its efficient-attention backward requires equal head counts).  Restore 4.45.2's
    # behaviour: K/V repeated, then SDPA.
    sdpa_attention.use_gqa_in_sdpa = lambda attention_mask, key: False
    # The reference records its dims with SDPA forced to the flash backend
    # (gen_node_tracing.py:22,68) and trains without forcing one, which on its testbed (torch 2.8,
    # RTX 3090) also selects flash.  torch 2.11 on B200 prefers cuDNN attention, which would
    # make the training graph differ from the recorded one; keep flash as the default.
    torch.backends.cuda.enable_cudnn_sdp(False)

    from grad_filter import token_filter  # the reference's extension
    from model.utils import token_filter_loss
    from gen_node_tracing import gen_node_tracing_with_model_with_dims

    assert os.path.abspath(token_filter.__file__).startswith(REF), token_filter.__file__
    assert "centrifuge_b200" not in sys.modules

    kw = dict(TINYLLAMA)
    kw["max_position_embeddings"] = max(kw["max_position_embeddings"], args.seq)
    if args.layers:
        kw["num_hidden_layers"] = args.layers
    # transformers 5.5 builds a KV cache in training forwards too and concatenates each layer's
    # K/V into it along the sequence (a CatBackward0 node the filter cannot shrink); 4.45.2 only
    # appended.  Training needs no cache: use_cache=False gives 4.45.2's autograd graph.
    kw["use_cache"] = False
    cfg = LlamaConfig(**kw)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(4321)
    model = LlamaForCausalLM(cfg).to(torch.bfloat16).to(dev)
    model.train()

    filtered = args.mode != "regular"
    attn_filter = args.mode == "centrifuge"
    dims = ""
    if attn_filter:
        # train.py:98-103: dims recorded on a probe batch before the optimizer wraps the model
        probe_bsz = 1 if args.mbs == 1 else 19
        dims = gen_node_tracing_with_model_with_dims(model, probe_bsz, 32 * 7, cfg.vocab_size, "")
        if not dims:
            raise RuntimeError("reference dims probe failed")
        model.zero_grad(set_to_none=True)

    opt = ZeroOneBF16(model, world, rank, lr=1e-4, betas=(0.9, 0.95), eps=1e-8,
                      weight_decay=0.0, clip=1.0)

    gen = torch.Generator().manual_seed(4321 + 1000003 * rank)

    def host_batch():
        ids = torch.randint(0, cfg.vocab_size, (args.mbs, args.seq), generator=gen).pin_memory()
        am = torch.ones(args.mbs, args.seq, dtype=torch.long).pin_memory()
        ref = torch.exp(1.0 + 0.5 * torch.randn(args.mbs, args.seq - 1, generator=gen))
        return ids, am, ref.tolist()  # the reference takes ref_loss as per-sample lists

    stats = {"filtering_ratio": []}

    def train_step(ids, am, ref_loss):
        """One micro-batch of the reference's Trainer.train_step (train.py:222-275)."""
        logits = model(ids, attention_mask=am).logits
        torch.cuda.synchronize()
        if filtered:
            loss, ref_mask = token_filter_loss(
                ids, logits, attention_mask=am, ref_loss=ref_loss, dropping_strategy="fixed",
                drop_rate=args.drop, is_left_padding=True, return_mask=True)
            all_token_loss = token_filter_loss(ids, logits, ref_loss=None, is_left_padding=True,
                                               return_mask=False)
        else:
            loss, ref_mask = token_filter_loss(ids, logits, attention_mask=am, ref_loss=None,
                                               is_left_padding=True, return_mask=True)
            all_token_loss = None
        torch.cuda.synchronize()
        if filtered:
            stats["filtering_ratio"].append(1 - float(ref_mask.sum()) / ref_mask.numel())
        if attn_filter:
            token_filter.ops.backward_filter_with_dims(loss, ref_mask, dims)
            torch.cuda.synchronize()
        lv = loss.item()
        if all_token_loss is not None:
            all_token_loss.item()
        (loss / args.ga).backward()
        torch.cuda.synchronize()
        opt.accumulate()
        return lv

    def optimizer_step(micro):
        total = 0.0
        for ids, am, ref in micro:
            total += train_step(ids, am, ref)
        opt.step()
        return total / len(micro)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- device-timed loop: token ids and attention masks staged on the device
    staged = []
    for _ in range(args.ga):
        ids, am, ref = host_batch()
        staged.append((ids.to(dev), am.to(dev), ref))
    # token_filter_loss zeroes the dropped positions of the attention mask in place (train.py:246
    # notes it), so every micro-batch gets its own mask, as the reference's data loader provides
    fresh = lambda: [(i, a.clone(), [list(r) for r in ref]) for i, a, ref in staged]  # noqa: E731
    for _ in range(args.warmup):
        optimizer_step(fresh())
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    batches = [fresh() for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        start.record()
        for b in batches:
            loss = optimizer_step(b)
        stop.record()
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = start.elapsed_time(stop)
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    tokens = world * args.ga * args.mbs * args.seq * args.steps
    value = tokens / (ms_max / 1000.0)

    # ---- end to end: every step copies its inputs host -> device and reads the loss back
    e2e = None
    if not args.no_e2e:
        host = [[host_batch() for _ in range(args.ga)] for _ in range(args.steps)]
        h2d = sum(i.nbytes + a.nbytes + 4 * len(r) * len(r[0]) for i, a, r in host[0])
        torch.cuda.synchronize()
        barrier()
        t0 = time.perf_counter()
        for step in range(args.steps):
            micro = [(i.to(dev, non_blocking=True), a.to(dev, non_blocking=True), r)
                     for i, a, r in host[step]]
            loss_val = optimizer_step(micro)
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        tw = torch.tensor([wall], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(tw, op=dist.ReduceOp.MAX)
        e2e = {"value": tokens / float(tw.item()), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 8 * args.ga * (2 if filtered else 1),
               "loss_last": loss_val}

    if rank == 0:
        so = sorted({line.split()[-1] for line in open("/proc/self/maps")
                     if line.rstrip().endswith(".so") and REPO in line})
        line = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (uniform token ids, LogNormal(1.0,0.5) ref_loss, random-init weights)",
            "config": {"model": "TinyLlama-1.1B", "global_batch": world * args.ga * args.mbs,
                       "micro_batch": args.mbs, "grad_accum": args.ga, "seq_len": args.seq,
                       "drop_rate": args.drop if filtered else 0.0, "mode": args.mode,
                       "parallelism": f"zero1-dp{world}",
                       "layers": cfg.num_hidden_layers,
                       "l2": "working set (weights + activations) far larger than L2"},
            "reference_path": "HF LlamaForCausalLM (sdpa) + model.utils.token_filter_loss + "
                              "token_filter.ops.backward_filter_with_dims (RESTORE_Q build)",
            "stand_ins": {"deepspeed_zero1_bf16": "flat bf16 params, fp32 grad accumulation, "
                                                  "NCCL reduce-scatter/all-gather, torch fused AdamW",
                          "lr_schedule": "constant",
                          "sdpa_backend": "flash (cuDNN SDPA disabled, as on the reference's "
                                          "testbed default)",
                          "transformers": "5.5 with K/V repeated before SDPA and use_cache=False, "
                                          "giving the autograd graph of the reference's pinned "
                                          "4.45.2"},
            "build": "baseline/build_ref.sh: unmodified sources, -include baseline/ref_compat.h "
                     "(torch 2.11 add_input_metadata arity), system g++",
            "filtering_ratio": (sum(stats["filtering_ratio"]) / len(stats["filtering_ratio"])
                                if stats["filtering_ratio"] else 0.0),
            "clocks": clocks.summary(), "e2e": e2e, "loss": loss,
            "native_so_loaded": so,
        }
        print(json.dumps(line), flush=True)
        if args.json_out:
            with open(args.json_out, "w") as f:
                json.dump(line, f, indent=1)
    if world > 1:
        barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
