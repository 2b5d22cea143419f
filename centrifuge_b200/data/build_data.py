"""Dataset building and caching for filtered training.

Reference: data/build_data.py.  Datasets are mixed from a registry of HuggingFace math/web
corpora (each mapped to a ``text`` column, instruction sets through a prompt template),
shuffled, optionally sub-selected, split train/valid, tokenised with overflow (and optionally
packed to exactly ``context_length`` tokens), optionally annotated with a per-token reference
loss, and saved to disk by rank 0; the other ranks wait on a barrier and load from disk.

Offline note: ``datasets.load_dataset`` needs either network access or a local HF cache.  The
pure functions here (packing, collation, prompt building) have no such dependency and are what
the tests exercise; ``--synthetic_data`` trains without any dataset.
"""
from __future__ import annotations

import os
from typing import Callable, Dict, List, Optional, Sequence

import numpy as np
import torch

DEFAULT_PROMPT = "Question: {instruction}\n\nAnswer: {response}"


# name -> (config, split, column renames, columns to drop, prompt, prompt entries)
DATASET_REGISTRY: Dict[str, dict] = {
    "meta-math/MetaMathQA": dict(split="train", rename={"query": "instruction"},
                                 drop=["type", "original_question"], prompt=DEFAULT_PROMPT,
                                 entries=["instruction", "response"]),
    "math-ai/StackMathQA": dict(config="stackmathqa1600k", split="train",
                                rename={"Q": "instruction", "A": "response"}, drop=["meta"],
                                prompt=DEFAULT_PROMPT, entries=["instruction", "response"]),
    "microsoft/orca-math-word-problems-200k": dict(
        split="train", rename={"question": "instruction", "answer": "response"},
        prompt=DEFAULT_PROMPT, entries=["instruction", "response"]),
    "TIGER-Lab/MathInstruct": dict(split="train", rename={"output": "response"}, drop=["source"],
                                   prompt=DEFAULT_PROMPT, entries=["instruction", "response"]),
    "open-web-math/open-web-math": dict(split="train", drop=["url", "date", "metadata"]),
    "DKYoon/SlimPajama-6B": dict(split="train", drop=["meta", "__index_level_0__"]),
    "hkust-nlp/dart-math-uniform": dict(split="train", rename={"query": "instruction"},
                                        prompt=DEFAULT_PROMPT, entries=["instruction", "response"]),
    "hkust-nlp/dart-math-hard": dict(split="train", rename={"query": "instruction"},
                                     prompt=DEFAULT_PROMPT, entries=["instruction", "response"]),
    "Vivacem/MMIQC": dict(split="train", rename={"output": "response"}, drop=["source"],
                          prompt=DEFAULT_PROMPT, entries=["instruction", "response"]),
    "lighteval/MATH": dict(splits=["train", "test"], drop=["level", "type"],
                           prompt="Question: {problem} Answer: {solution}",
                           entries=["problem", "solution"]),
    "nvidia/OpenMathInstruct-2": dict(split="train_5M",
                                      prompt="Question: {problem} Answer: {generated_solution}",
                                      entries=["problem", "generated_solution"]),
}


def build_prompt(batch: dict, prompt: str, entries: Sequence[str],
                 entry_func: Callable[[dict], dict] = lambda x: x) -> dict:
    n = len(batch[entries[0]])
    batch["prompt"] = [prompt.format(**entry_func({e: batch[e][i] for e in entries}))
                       for i in range(n)]
    return batch


def build_instruct(ds, prompt: str = DEFAULT_PROMPT, entries=("instruction", "response"),
                   entry_func=lambda x: x, num_proc: Optional[int] = None):
    return ds.map(build_prompt, fn_kwargs=dict(prompt=prompt, entries=list(entries),
                                               entry_func=entry_func),
                  batched=True, batch_size=1000, num_proc=num_proc,
                  remove_columns=list(entries)).rename_column("prompt", "text")


def load_one(name: str):
    from datasets import concatenate_datasets, load_dataset
    spec = DATASET_REGISTRY.get(name)
    if spec is None:
        raise KeyError(f"unknown dataset {name!r}; known: {sorted(DATASET_REGISTRY)}")
    splits = spec.get("splits", [spec.get("split", "train")])
    parts = [load_dataset(name, spec.get("config"), split=s) for s in splits]
    ds = concatenate_datasets(parts) if len(parts) > 1 else parts[0]
    drop = [c for c in spec.get("drop", []) if c in ds.column_names]
    if drop:
        ds = ds.remove_columns(drop)
    if spec.get("rename"):
        ds = ds.rename_columns({k: v for k, v in spec["rename"].items() if k in ds.column_names})
    if "prompt" in spec:
        ds = build_instruct(ds, spec["prompt"], spec["entries"])
    return ds


def build_pretrain_data(datasets: Sequence[str], train_val_split=(0.999, 0.001), seed=None,
                        data_select_ratio: float = 1.0, data_select_strategy: str = "random"):
    from datasets import DatasetDict, concatenate_datasets
    ds = concatenate_datasets([load_one(n) for n in datasets]).shuffle(seed=seed)
    assert 0 < data_select_ratio <= 1
    if data_select_ratio < 1:
        if data_select_strategy != "random":
            raise ValueError("Unknown data selection strategy")
        ds = ds.select(range(int(len(ds) * data_select_ratio)))
    n_train = int(len(ds) * train_val_split[0])
    return DatasetDict({"train": ds.select(range(n_train)),
                        "valid": ds.select(range(n_train, len(ds)))})


def pack_token_ids(seqs: Sequence[Sequence[int]], context_length: int):
    """Concatenate token sequences and cut them into rows of exactly ``context_length``
    (the last row may be shorter).  Returns ``(rows, lengths, sample_map)`` where
    ``sample_map[i]`` is the index of the sequence in which row ``i`` ends
    (data/build_data.py:290-320)."""
    rows, lengths, smap = [], [], []
    cur: List[int] = []
    i, start = 0, 0
    while i < len(seqs):
        need = context_length - len(cur)
        piece = seqs[i][start:start + need]
        cur.extend(piece)
        if need >= len(seqs[i]) - start:
            i, start = i + 1, 0
        else:
            start += need
        if len(cur) == context_length or i == len(seqs):
            rows.append(cur)
            lengths.append(len(cur))
            smap.append(i)
            cur = []
    assert sum(lengths) == sum(len(s) for s in seqs)
    return rows, lengths, smap


def tokenize_batch(texts: Sequence[str], tokenizer, context_length: int, add_eos: bool = False,
                   packing: bool = False) -> dict:
    if add_eos:
        texts = [t + tokenizer.eos_token for t in texts]
    out = tokenizer(list(texts), max_length=context_length, truncation=True,
                    return_overflowing_tokens=True, return_length=True)
    if packing:
        rows, lengths, smap = pack_token_ids(out["input_ids"], context_length)
        return {"input_ids": rows, "length": lengths, "overflow_to_sample_mapping": smap}
    return dict(out)


def collate_fn(batch: List[dict]) -> dict:
    """Left-pad ``input_ids`` with 0 and ``attention_mask`` with 0; carry ``ref_loss``,
    ``length`` and ``text`` through (model/utils.py:269-286)."""
    longest = max(len(x["input_ids"]) for x in batch)
    ids = np.stack([[0] * (longest - len(x["input_ids"])) + list(x["input_ids"]) for x in batch])
    masks = []
    for x in batch:
        m = x.get("attention_mask") or [1] * len(x["input_ids"])
        masks.append([0] * (longest - len(m)) + list(m))
    out = {"input_ids": torch.from_numpy(ids).long(),
           "attention_mask": torch.from_numpy(np.stack(masks)).long()}
    for key in ("text", "ref_loss", "length"):
        if key in batch[0]:
            out[key] = [x[key] for x in batch]
    return out


def create_synthetic_dataset(vocab_size: int, context_length: int, num_samples: int,
                             seed: int = 0):
    """HF ``Dataset`` of random ids, all-ones mask, zero ref_loss (data/build_data.py:15-25)."""
    from datasets import Dataset
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab_size, (num_samples, context_length), generator=g).tolist()
    return Dataset.from_dict({
        "input_ids": ids,
        "attention_mask": [[1] * context_length for _ in range(num_samples)],
        "ref_loss": [[0.0] * (context_length - 1) for _ in range(num_samples)],
        "length": [context_length] * num_samples,
    })


def build_tokenized_datasets(args, ref_loss_fn: Optional[Callable] = None):
    """Load the tokenised dataset from ``args.data_cache_dir`` or build it on rank 0.

    ``ref_loss_fn(list_of_token_id_lists) -> list_of_loss_lists`` annotates each row with a
    reference loss when ``args.pre_compute_ref`` is set (HF model, vLLM, socket or n-gram
    backends; see :mod:`centrifuge_b200.data.ref_server`).
    """
    import torch.distributed as dist
    from datasets import load_from_disk
    try:
        return load_from_disk(args.data_cache_dir)
    except Exception:
        pass
    rank0 = not dist.is_initialized() or dist.get_rank() == 0
    if rank0:
        from transformers import AutoTokenizer
        raw = build_pretrain_data(args.datasets.split(","), (args.train_ratio, 1 - args.train_ratio),
                                  args.random_seed, args.data_select_ratio,
                                  args.data_select_strategy)
        tok = AutoTokenizer.from_pretrained(args.model_path)

        def fn(batch):
            out = tokenize_batch(batch["text"], tok, args.context_length, args.add_eos_token,
                                 args.packing_samples)
            if args.pre_compute_ref and ref_loss_fn is not None:
                out["ref_loss"] = []
                for i in range(0, len(out["input_ids"]), 8):
                    out["ref_loss"] += ref_loss_fn(out["input_ids"][i:i + 8])
            return out

        ds = raw.map(fn, batched=True, batch_size=10000, remove_columns=raw["train"].column_names,
                     num_proc=1 if args.pre_compute_ref else max(1, (os.cpu_count() or 2) // 2))
        ds.save_to_disk(args.data_cache_dir)
    if dist.is_initialized():
        dist.barrier()
    return load_from_disk(args.data_cache_dir)
