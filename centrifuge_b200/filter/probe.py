"""Autograd probe: which backward node types does a model's filtered loss produce?

Offline onboarding step 1 (reference grad_filter/add_torch_native_model.py:77-174): build the
model from its config with random weights (bf16 unless on CPU), run a training-mode forward,
the filtered loss with a fixed 50% drop, and collect the names of every node in the backward
graph.  The names are merged (append-only, sorted, with a ``.bak`` of the previous file) into
``target_node_names.yaml``, from which :mod:`centrifuge_b200.filter.codegen` generates the
rewriter's node handlers.
"""
from __future__ import annotations

import os
import shutil
from collections import deque
from typing import Iterable, List, Optional

import torch
import yaml


def collect_node_names_py(loss: torch.Tensor) -> List[str]:
    """Names of all nodes reachable from ``loss.grad_fn`` (Python traversal; the C++ op
    ``token_filter::collect_node_names`` returns the same set)."""
    seen, names = set(), set()
    q = deque([loss.grad_fn])
    while q:
        fn = q.popleft()
        if fn is None or fn in seen:
            continue
        seen.add(fn)
        names.add(type(fn).__name__ if type(fn).__name__ != "AccumulateGrad"
                  else "torch::autograd::AccumulateGrad")
        for nxt, _ in getattr(fn, "next_functions", ()):
            if nxt is not None:
                q.append(nxt)
    return sorted(names)


def align_seq_len(n: int, multiple: int = 8) -> int:
    return (n + multiple - 1) // multiple * multiple


def build_hf_model(model_path_or_config, attn_impl: str = "sdpa", device: str = "cpu",
                   dtype=None):
    from transformers import AutoConfig, AutoModelForCausalLM, LlamaConfig as HFLlamaConfig
    if isinstance(model_path_or_config, str) and os.path.isdir(model_path_or_config):
        cfg = AutoConfig.from_pretrained(model_path_or_config)
    elif isinstance(model_path_or_config, dict):
        cfg = HFLlamaConfig(**model_path_or_config)
    else:
        cfg = model_path_or_config
    cfg._attn_implementation = attn_impl
    cfg.use_cache = False  # training graph: no KV-cache concatenation
    model = AutoModelForCausalLM.from_config(cfg)
    dtype = dtype or (torch.bfloat16 if device != "cpu" else torch.float32)
    return model.to(device=device, dtype=dtype).train()


def probe(model, seq_len: int = 224, batch: int = 1, drop_rate: float = 0.5,
          device: str = "cpu", seed: int = 0) -> List[str]:
    from ..loss import token_filter_loss
    g = torch.Generator().manual_seed(seed)
    vocab = model.config.vocab_size
    seq_len = align_seq_len(seq_len)
    ids = torch.randint(0, vocab, (batch, seq_len), generator=g).to(device)
    mask = torch.ones(batch, seq_len, dtype=torch.long, device=device)
    ref = torch.randn(batch, seq_len - 1, generator=g).to(device)
    logits = model(input_ids=ids).logits
    loss, _ = token_filter_loss(ids, logits, mask, ref, "fixed", drop_rate, True, True)
    return collect_node_names_py(loss)


def write_yaml(names: Iterable[str], path: str) -> List[str]:
    """Merge ``names`` into the yaml (append-only, sorted); keeps ``path + '.bak'``."""
    old: List[str] = []
    if os.path.exists(path):
        with open(path) as f:
            old = (yaml.safe_load(f) or {}).get("target_node_names", []) or []
        shutil.copyfile(path, path + ".bak")
    merged = sorted(set(old) | set(names))
    with open(path, "w") as f:
        yaml.safe_dump({"target_node_names": merged}, f, default_flow_style=False)
    return merged


def main(argv: Optional[List[str]] = None):
    import argparse
    from ..config import get_model_config
    ap = argparse.ArgumentParser(description="probe a model's backward node types")
    ap.add_argument("--model_path", default="tiny")
    ap.add_argument("--context_length", type=int, default=224)
    ap.add_argument("--attn_impl", default="sdpa", choices=["eager", "sdpa", "flash_attention_2"])
    ap.add_argument("--use_lora", action="store_true")
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--yaml", default=None)
    a = ap.parse_args(argv)
    try:
        cfg = get_model_config(a.model_path).to_hf_dict()
    except KeyError:
        cfg = a.model_path
    model = build_hf_model(cfg, a.attn_impl, a.device)
    if a.use_lora:
        from ..models.lora import apply_lora
        apply_lora(model, r=64, alpha=128, dropout=0.1)
    names = probe(model, a.context_length, device=a.device)
    from .codegen import DEFAULT_YAML
    path = a.yaml or DEFAULT_YAML
    merged = write_yaml(names, path)
    print(f"{len(names)} node types probed; {len(merged)} in {path}")


if __name__ == "__main__":
    main()
