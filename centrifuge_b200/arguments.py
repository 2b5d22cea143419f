"""Command-line flags of the training entry points.

Same flag names, groups, choices and defaults as the reference (arguments.py:9-91), so existing
launch scripts keep working, plus the B200-native options (model implementation, ZeRO stage,
tensor / sequence / pipeline parallelism).  ``get_cache_dir`` names the model and data cache
directories from an md5 of the identifying arguments (data/build_data.py:28-47).
"""
from __future__ import annotations

import argparse
import copy
import hashlib
import os
import sys
from typing import List, Optional

UN_IDENTIFY_ARGS = [
    "ref_socket_hosts", "ref_socket_ports", "vllm_url", "pre_compute_ref", "local_rank",
    "model_cache_dir", "data_cache_dir", "output_dir", "attn_impl",
]


def build_parser() -> argparse.ArgumentParser:
    ap = argparse.ArgumentParser(description="centrifuge_b200 filtered training")
    ap.add_argument("--local_rank", type=int, default=-1,
                    help="local rank passed from the distributed launcher")
    ap.add_argument("--task", type=str, default="train",
                    choices=["gen-data", "train", "eff-benchmark", "param-search"])

    g = ap.add_argument_group("Model and Data")
    g.add_argument("--datasets", type=str, default="open-web-math/open-web-math")
    g.add_argument("--dataset_path", type=str, help="path of a previously built dataset")
    g.add_argument("--model_path", type=str, default="TinyLlama/TinyLlama_v1.1")
    g.add_argument("--output_dir", type=str, default="debug")
    g.add_argument("--model_cache_dir", type=str, default=None, help="named automatically")
    g.add_argument("--data_cache_dir", type=str, default=None, help="named automatically")
    g.add_argument("--data_select_ratio", type=float, default=1.0)
    g.add_argument("--data_select_strategy", type=str, default="random")
    g.add_argument("--add_eos_token", action="store_true", default=False)
    g.add_argument("--packing_samples", action="store_true", default=False)
    g.add_argument("--use_lora", action="store_true", default=False)
    g.add_argument("--attn_impl", type=str, default="flash_attention_2",
                   choices=["eager", "flash_attention_2", "sdpa"])

    g = ap.add_argument_group("Training")
    g.add_argument("--batch_size", type=int, default=512)
    g.add_argument("--micro_batch_size", type=int, default=1)
    g.add_argument("--weight_decay", type=float, default=1e-2)
    g.add_argument("--context_length", type=int, default=2048)
    g.add_argument("--random_seed", type=int, default=1234)
    g.add_argument("--epochs", type=int, default=1)
    g.add_argument("--learning_rate", type=float, default=6e-5)
    g.add_argument("--use_layer_lr", action="store_true", default=False,
                   help="different learning rates for different layers")
    g.add_argument("--layer_lr_decay", type=float, default=1.0,
                   help="learning-rate decay from output to input")
    g.add_argument("--eval_steps", type=int, default=1000)
    g.add_argument("--gradient_accumulation_steps", type=int,
                   help="calculated automatically from batch / micro-batch / world size")
    g.add_argument("--train_ratio", type=float, default=0.999)
    g.add_argument("--save_steps", type=int, default=100)

    g = ap.add_argument_group("Token Dropping")
    g.add_argument("--ref_model_backend", type=str, default="none",
                   choices=["hf", "vllm", "socket", "none", "self"])
    g.add_argument("--ref_socket_hosts", type=str, default="None")
    g.add_argument("--ref_socket_ports", type=str, default="None")
    g.add_argument("--vllm_url", type=str, default="None")
    g.add_argument("--ref_model_path", type=str, default="None")
    g.add_argument("--dropping_strategy", type=str, default="none",
                   choices=["none", "fixed", "positive", "dynamic", "peaking", "less_ref", "self"])
    g.add_argument("--drop_rate", type=float, default=0)
    g.add_argument("--pre_compute_ref", action="store_true", default=False)
    g.add_argument("--attn_filter", action="store_true", default=False,
                   help="rewrite the backward to run on kept tokens (backward_filter)")
    g.add_argument("--forward_filter", action="store_true", default=False,
                   help="accepted for compatibility; not implemented (as in the reference)")
    g.add_argument("--filter_opt", default=0, type=int,
                   help="accepted for compatibility (0: no opt, 1: MLP, 2: +Attn MM, 3: +Attn out)")

    g = ap.add_argument_group("B200 runtime")
    g.add_argument("--model_impl", type=str, default="native", choices=["native", "hf"],
                   help="native: fused sm_100a Llama; hf: HuggingFace model + graph rewriter")
    g.add_argument("--zero_stage", type=int, default=2, choices=[1, 2])
    g.add_argument("--tensor_parallel_size", type=int, default=1)
    g.add_argument("--pipeline_parallel_size", type=int, default=1)
    g.add_argument("--sequence_parallel", action="store_true", default=False)
    g.add_argument("--num_microbatches", type=int, default=None,
                   help="pipeline micro-batches per step (default: gradient accumulation)")
    g.add_argument("--grad_reducer", type=str, default="auto", choices=["auto", "nccl", "symm"])
    g.add_argument("--grad_mode", type=str, default="ring", choices=["ring", "full"],
                   help="ZeRO-2 gradients: ring = partitioned (bucket slots reduce-scattered "
                        "every micro-batch), full = full local buffer reduced once per step")
    g.add_argument("--max_steps", type=int, default=None)
    g.add_argument("--log_file", type=str, default=None, help="JSONL metrics file")
    g.add_argument("--synthetic_data", action="store_true", default=False,
                   help="uniform token ids + LogNormal(1, 0.5) ref_loss instead of datasets")

    g = ap.add_argument_group("Utils")
    g.add_argument("--un_identify_args", required=False,
                   default=UN_IDENTIFY_ARGS + ["un_identify_args"], nargs="+")
    return ap


def parse_args(argv: Optional[List[str]] = None, return_parsed: bool = True):
    ap = build_parser()
    return ap.parse_args(argv) if return_parsed else ap


def cache_root() -> str:
    return os.environ.get("HF_HOME", os.path.join(os.path.expanduser("~"), ".cache", "huggingface"))


def get_cache_dir(args, create: bool = True):
    """``(model_cache_dir, data_cache_dir)`` named from the identifying arguments."""
    d = vars(copy.deepcopy(args))
    for a in getattr(args, "un_identify_args", UN_IDENTIFY_ARGS):
        d.pop(a, None)
    md5 = hashlib.md5(str(d).encode()).hexdigest()
    root = os.path.join(cache_root(), "token_dropping")
    model_dir = args.model_cache_dir or os.path.join(root, f"{args.output_dir}_{md5}")
    data_dir = args.data_cache_dir or os.path.join(
        root, "data", args.datasets.replace(",", "-").replace("/", "-") +
        f"_{args.data_select_strategy}_{args.data_select_ratio}_{args.random_seed}"
        f"_{args.train_ratio}_{args.context_length}")
    if args.data_cache_dir is None:
        if args.add_eos_token:
            data_dir += "_weos"
        if args.packing_samples:
            data_dir += "_pack"
        if args.pre_compute_ref:
            data_dir += "_wref"
    if create:
        os.makedirs(model_dir, exist_ok=True)
        os.makedirs(data_dir, exist_ok=True)
    args.model_cache_dir, args.data_cache_dir = model_dir, data_dir
    return model_dir, data_dir
