"""Training entry point (``python train.py ...`` / ``torchrun ... train.py ...``).

Tasks (reference train.py:380-464): ``train`` (datasets or ``--synthetic_data``),
``eff-benchmark`` (synthetic batches, 12 optimizer steps, first 2 are warm-up, per-phase
timings to ``batch_time_{rank}.json``), ``gen-data`` (build and cache the tokenised dataset,
optionally with pre-computed reference losses) and ``param-search`` (stops after 1000 steps).

Model implementations:
* ``--model_impl native`` (default): the fused sm_100a Llama with ZeRO-1/2 (``--zero_stage``),
  filtered by attaching the selection mask to its backward node.
* ``--model_impl hf``: any HuggingFace causal LM (optionally with LoRA adapters); the backward
  is filtered by the C++ graph rewriter with dims recorded once on a probe batch (S=224) and
  replayed every micro-batch, as the reference does (train.py:97-103, 259-269).
"""
from __future__ import annotations

import datetime
import json
import os
import sys
import time
from typing import Iterator, List, Optional

import torch
import torch.distributed as dist

from .arguments import get_cache_dir, parse_args
from .config import get_model_config
from .data.synthetic import Batch, SyntheticTokenData
from .loss import token_filter_loss
from .utils.metrics import MetricsWriter
from .utils.schedule import WarmupCosineLR
from .utils.timer import StepTimer

EFF_BENCH_ITERS = 12  # 2 warm-up + 10 timed (reference train.py:41)


def init_distributed():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if torch.cuda.is_available():
        torch.cuda.set_device(local)
    if world > 1 and not dist.is_initialized():
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = dict(timeout=datetime.timedelta(minutes=30))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, **kw)
    return world, rank, local


def _batches_from_dataset(ds, micro_bs: int, rank: int, world: int, seed: int) -> Iterator[Batch]:
    from torch.utils.data import DataLoader, DistributedSampler

    from .data.build_data import collate_fn
    sampler = DistributedSampler(ds, num_replicas=world, rank=rank, shuffle=False) if world > 1 else None
    for b in DataLoader(ds, batch_size=micro_bs, collate_fn=collate_fn, sampler=sampler):
        ref = None
        if "ref_loss" in b:
            S = b["input_ids"].shape[1]
            ref = torch.tensor([[0.0] * (S - 1 - len(r)) + list(r) for r in b["ref_loss"]])
        yield Batch(b["input_ids"], ref if ref is not None else torch.zeros(
            b["input_ids"].shape[0], b["input_ids"].shape[1] - 1), b["attention_mask"])


class NativeRunner:
    """Native B200 model + ZeRO optimizer + filtered trainer."""

    def __init__(self, args, world, rank, device):
        from .models.llama import NativeLlamaForCausalLM
        from .parallel.zero import ZeroAdamW
        from .trainer import Trainer
        self.cfg = get_model_config(args.model_path)
        self.cfg.max_position_embeddings = max(self.cfg.max_position_embeddings, args.context_length)
        self.model = NativeLlamaForCausalLM(self.cfg, device=device, seed=args.random_seed,
                                            pad_to=world)
        ckpt = args.model_path if os.path.isdir(args.model_path) else None
        if ckpt and any(f.endswith(".safetensors") for f in os.listdir(ckpt)):
            from .utils.checkpoint import load_model_
            load_model_(self.model, ckpt)
        group = dist.group.WORLD if world > 1 else None
        reducer = None
        if world > 1 and args.grad_reducer in ("auto", "symm") and device.type == "cuda":
            try:
                from .parallel.symm import SymmReducer
                reducer = SymmReducer.create(self.model.flat, group,
                                             ring=args.grad_mode == "ring" and args.zero_stage == 2)
            except Exception:
                if args.grad_reducer == "symm":
                    raise
        self.opt = ZeroAdamW(self.model.flat, group=group, stage=args.zero_stage,
                             lr=args.learning_rate, betas=(0.9, 0.95), eps=1e-8,
                             weight_decay=args.weight_decay, grad_clip=1.0, reducer=reducer,
                             grad_mode=args.grad_mode if args.zero_stage == 2 else "full")
        drop = args.drop_rate if args.dropping_strategy not in ("none", None) else 0.0
        self.trainer = Trainer(self.model, self.opt, drop_rate=drop,
                               strategy=args.dropping_strategy, grad_accum=args.gradient_accumulation_steps,
                               world_size=world)

    def set_lr(self, lr):
        self.opt.lr = lr

    def step(self, batches: List[Batch]) -> torch.Tensor:
        return self.trainer.train_step(batches)

    @torch.no_grad()
    def eval_loss(self, batches: List[Batch]) -> float:
        tot, n = 0.0, 0
        for b in batches:
            b = b.to(self.model.device)
            out = self.model(b.input_ids)
            tot += float(out.token_loss.mean())
            n += 1
        return tot / max(1, n)

    def save(self, out_dir: str, rank: int, client_state: dict) -> None:
        from .utils.checkpoint import save_model, save_training_state
        if rank == 0:
            save_model(self.model, out_dir)
        save_training_state(out_dir, rank, self.opt.state_dict(), client_state)

    def restore(self, out_dir: str, rank: int) -> Optional[dict]:
        from .utils.checkpoint import load_training_state
        try:
            shard, client = load_training_state(out_dir, rank)
        except FileNotFoundError:
            return None
        self.opt.load_state_dict(shard)
        return client


class HFRunner:
    """HuggingFace model filtered by the graph rewriter (generic path)."""

    def __init__(self, args, world, rank, device):
        from .filter import backward_filter_with_dims
        from .filter.probe import build_hf_model
        try:
            cfg = get_model_config(args.model_path).to_hf_dict()
        except KeyError:
            cfg = args.model_path
        dtype = torch.bfloat16 if device.type == "cuda" else torch.float32
        self.model = build_hf_model(cfg, "sdpa" if args.attn_impl != "eager" else "eager",
                                    str(device), dtype)
        if args.use_lora:
            from .models.lora import apply_lora
            apply_lora(self.model)
        self.params = [p for p in self.model.parameters() if p.requires_grad]
        if world > 1:
            self.model = torch.nn.parallel.DistributedDataParallel(
                self.model, device_ids=[device.index] if device.type == "cuda" else None)
        self.opt = torch.optim.AdamW(self.params, lr=args.learning_rate, betas=(0.9, 0.95),
                                     weight_decay=args.weight_decay)
        self.args, self.world, self.device = args, world, device
        self.ga = args.gradient_accumulation_steps
        self.drop = args.drop_rate if args.dropping_strategy not in ("none", None) else 0.0
        self.dims = ""
        self._bf = backward_filter_with_dims
        if args.attn_filter and self.drop > 0:
            self.dims = self._probe_dims()

    def _probe_dims(self) -> str:
        """Record the dims on a probe batch whose sizes do not collide with model dims."""
        vocab = self._core().config.vocab_size
        S = 224
        B = 1 if self.args.micro_batch_size == 1 else 19
        ids = torch.randint(0, vocab, (B, S), device=self.device)
        ref = torch.randn(B, S - 1, device=self.device)
        logits = self.model(input_ids=ids).logits
        loss, mask = token_filter_loss(ids, logits, torch.ones(B, S, dtype=torch.long, device=self.device),
                                       ref, "fixed", 0.5, True, True)
        dims = self._bf(loss, mask, "")
        loss.backward()
        self.opt.zero_grad(set_to_none=True)
        return dims

    def _core(self):
        return self.model.module if hasattr(self.model, "module") else self.model

    def set_lr(self, lr):
        for g in self.opt.param_groups:
            g["lr"] = lr

    def step(self, batches: List[Batch]) -> torch.Tensor:
        total = torch.zeros((), device=self.device)
        for b in batches:
            b = b.to(self.device)
            B, S = b.input_ids.shape
            mask = b.attention_mask.clone() if b.attention_mask is not None else torch.ones(
                B, S, dtype=torch.long, device=self.device)
            logits = self.model(input_ids=b.input_ids, attention_mask=mask).logits
            if self.drop > 0:
                loss, mask = token_filter_loss(b.input_ids, logits, mask, b.ref_loss,
                                               self.args.dropping_strategy, self.drop, True, True)
                if self.args.attn_filter:
                    try:
                        self._bf(loss, mask, self.dims)
                    except RuntimeError as e:  # reference behaviour: skip the micro-step
                        print(f"backward filter failed ({e}); skipping the micro-batch")
                        continue
            else:
                loss = token_filter_loss(b.input_ids, logits, mask, None, None, None, True)
            (loss / self.ga).backward()
            total += loss.detach()
        torch.nn.utils.clip_grad_norm_(self.params, 1.0)
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return total / self.ga

    @torch.no_grad()
    def eval_loss(self, batches):
        tot = 0.0
        for b in batches:
            b = b.to(self.device)
            logits = self.model(input_ids=b.input_ids).logits
            tot += float(token_filter_loss(b.input_ids, logits, None, None, None, None, True))
        return tot / max(1, len(batches))

    def save(self, out_dir, rank, client_state):
        if rank == 0:
            self._core().save_pretrained(out_dir, safe_serialization=True)
        os.makedirs(os.path.join(out_dir, "training_states"), exist_ok=True)
        torch.save({"opt": self.opt.state_dict(), "client": client_state},
                   os.path.join(out_dir, "training_states", f"hf_rank{rank}.pt"))

    def restore(self, out_dir, rank):
        p = os.path.join(out_dir, "training_states", f"hf_rank{rank}.pt")
        if not os.path.exists(p):
            return None
        st = torch.load(p, map_location="cpu")
        self.opt.load_state_dict(st["opt"])
        return st["client"]


def main(argv: Optional[List[str]] = None) -> int:
    args = parse_args(argv)
    world, rank, local = init_distributed()
    torch.manual_seed(args.random_seed)
    device = torch.device("cuda", local) if torch.cuda.is_available() else torch.device("cpu")
    if args.gradient_accumulation_steps is None:
        args.gradient_accumulation_steps = max(1, args.batch_size // args.micro_batch_size // world)
    get_cache_dir(args)
    out_dir = args.model_cache_dir
    if rank == 0:
        with open(os.path.join(out_dir, "args.json"), "w") as f:
            json.dump(vars(args), f, default=str)
    ga = args.gradient_accumulation_steps

    synthetic = args.synthetic_data or args.task == "eff-benchmark"
    cfg = get_model_config(args.model_path) if not os.path.isdir(args.model_path) else None
    vocab = (cfg or get_model_config(args.model_path)).vocab_size
    if synthetic:
        data = SyntheticTokenData(vocab, args.micro_batch_size, args.context_length,
                                  seed=args.random_seed, rank=rank,
                                  zero_ref=args.task == "eff-benchmark")
        micro_iter: Iterator[Batch] = iter(data)
        eval_batches = [data.sample() for _ in range(2)]
    else:
        from .data.build_data import build_tokenized_datasets
        ds = build_tokenized_datasets(args)
        if args.task == "gen-data":
            return 0
        micro_iter = _batches_from_dataset(ds["train"], args.micro_batch_size, rank, world,
                                           args.random_seed)
        eval_batches = list(_batches_from_dataset(ds["valid"], 8, 0, 1, args.random_seed))[:8]
    if args.task == "gen-data":
        return 0

    runner = (NativeRunner if args.model_impl == "native" else HFRunner)(args, world, rank, device)
    metrics = MetricsWriter(out_dir, rank)
    timer = StepTimer(os.path.join(out_dir, f"batch_time_{rank}.json"), warmup=2)
    client = runner.restore(out_dir, rank) if args.task == "train" else None
    completed = client["completed_steps"] if client else 0
    if args.max_steps:
        total_steps = args.max_steps
    elif args.task == "eff-benchmark":
        total_steps = EFF_BENCH_ITERS
    elif args.task == "param-search":
        total_steps = 1000
    else:
        total_steps = 10 ** 9 if synthetic else len(ds["train"]) * args.epochs // args.batch_size
    sched = WarmupCosineLR(args.learning_rate, total_steps, total_steps // 20)
    # skip micro-batches already consumed before the restart
    for _ in range(completed * ga):
        next(micro_iter, None)
    tokens_per_step = world * ga * args.micro_batch_size * args.context_length
    while completed < total_steps:
        batches = []
        for _ in range(ga):
            b = next(micro_iter, None)
            if b is None:
                break
            batches.append(b)
        if len(batches) < ga:
            break
        runner.set_lr(sched(completed))
        timer.start()
        loss = runner.step(batches)
        timer.record("step")
        rec = timer.end()
        completed += 1
        if rank == 0:
            loss_v = float(loss)
            tps = tokens_per_step / (rec.get("total", rec["wall_total"]) / 1000.0)
            print(json.dumps({"steps": completed, "loss/train": loss_v, "lr": sched(completed - 1),
                              "tokens_per_s": tps}), flush=True)
            metrics.log(completed, {"train/loss/train": loss_v, "train/tokens_per_s": tps,
                                    "train/timer/total": rec.get("total", rec["wall_total"])})
        if args.task == "train" and completed % args.eval_steps == 0 and rank == 0:
            el = runner.eval_loss(eval_batches)
            metrics.log(completed, {"eval/loss": el, "eval/perplexity": float(torch.exp(torch.tensor(el)))})
        if args.task == "train" and completed % args.save_steps == 0:
            runner.save(out_dir, rank, {"step": completed * ga, "completed_steps": completed})
    if args.task == "train":
        runner.save(out_dir, rank, {"step": completed * ga, "completed_steps": completed})
    metrics.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
