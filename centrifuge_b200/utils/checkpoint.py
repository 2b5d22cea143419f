"""Checkpoints in HuggingFace Llama layout plus resumable training state.

* Model weights: ``model.safetensors`` (or sharded ``model-XXXXX-of-YYYYY.safetensors`` with an
  index) with HF-Llama state-dict names and ``config.json`` -- what the reference writes with
  ``save_pretrained`` (train.py:328-331), so checkpoints load in ``transformers``.
* Training state: ``training_states/`` with one ``optim_rank{r}.pt`` per data-parallel rank
  (the rank's ZeRO shard of fp32 master weights and Adam moments) and ``client_state.json``
  holding ``{"step", "completed_steps"}`` -- the content of the reference's DeepSpeed
  ``save_checkpoint(tag="train", client_state=...)`` (train.py:333-345).

The native models keep fused weights (``wqkv = [q; k; v]``, ``wgu = [gate; up]``); the
converters below split and join them.  Tensor-parallel shards are gathered to the HF layout on
save and re-sharded on load (see :mod:`centrifuge_b200.parallel.tensor_parallel`).
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterable, Optional

import torch

from ..config import LlamaConfig


def native_to_hf(cfg: LlamaConfig, params: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
    """Map native fused names (``layers.{i}.wqkv`` ...) to HF names; missing entries skipped."""
    H, F = cfg.hidden_size, cfg.intermediate_size
    q, kv = cfg.q_size, cfg.kv_size
    out = {}
    for name, t in params.items():
        if name == "embed":
            out["model.embed_tokens.weight"] = t
        elif name == "norm":
            out["model.norm.weight"] = t
        elif name == "lm_head":
            out["lm_head.weight"] = t
        elif name.startswith("layers."):
            _, i, w = name.split(".")
            p = f"model.layers.{i}."
            if w == "wqkv":
                out[p + "self_attn.q_proj.weight"] = t[:q]
                out[p + "self_attn.k_proj.weight"] = t[q:q + kv]
                out[p + "self_attn.v_proj.weight"] = t[q + kv:q + 2 * kv]
            elif w == "wo":
                out[p + "self_attn.o_proj.weight"] = t
            elif w == "wgu":
                out[p + "mlp.gate_proj.weight"] = t[:F]
                out[p + "mlp.up_proj.weight"] = t[F:2 * F]
            elif w == "wd":
                out[p + "mlp.down_proj.weight"] = t
            elif w == "ln1":
                out[p + "input_layernorm.weight"] = t
            elif w == "ln2":
                out[p + "post_attention_layernorm.weight"] = t
    return out


def hf_to_native_(cfg: LlamaConfig, hf: Dict[str, torch.Tensor],
                  params: Dict[str, torch.Tensor]) -> None:
    """Copy HF-named tensors into the native (fused) parameter views that exist in ``params``."""
    q, kv, F = cfg.q_size, cfg.kv_size, cfg.intermediate_size
    for name, dst in params.items():
        with torch.no_grad():
            if name == "embed":
                dst.copy_(hf["model.embed_tokens.weight"])
            elif name == "norm":
                dst.copy_(hf["model.norm.weight"])
            elif name == "lm_head":
                dst.copy_(hf["lm_head.weight"])
            else:
                _, i, w = name.split(".")
                p = f"model.layers.{i}."
                if w == "wqkv":
                    dst[:q].copy_(hf[p + "self_attn.q_proj.weight"])
                    dst[q:q + kv].copy_(hf[p + "self_attn.k_proj.weight"])
                    dst[q + kv:].copy_(hf[p + "self_attn.v_proj.weight"])
                elif w == "wo":
                    dst.copy_(hf[p + "self_attn.o_proj.weight"])
                elif w == "wgu":
                    dst[:F].copy_(hf[p + "mlp.gate_proj.weight"])
                    dst[F:].copy_(hf[p + "mlp.up_proj.weight"])
                elif w == "wd":
                    dst.copy_(hf[p + "mlp.down_proj.weight"])
                elif w == "ln1":
                    dst.copy_(hf[p + "input_layernorm.weight"])
                elif w == "ln2":
                    dst.copy_(hf[p + "post_attention_layernorm.weight"])


def save_pretrained(path: str, cfg: LlamaConfig, hf_state: Dict[str, torch.Tensor],
                    max_shard_bytes: int = 5 * 1024 ** 3) -> None:
    """Write ``config.json`` and safetensors shards of an HF-named state dict."""
    from safetensors.torch import save_file
    os.makedirs(path, exist_ok=True)
    cfg.save(os.path.join(path, "config.json"))
    items = [(k, v.detach().to("cpu").contiguous()) for k, v in hf_state.items()]
    shards, cur, size = [], {}, 0
    for k, v in items:
        nb = v.numel() * v.element_size()
        if cur and size + nb > max_shard_bytes:
            shards.append(cur)
            cur, size = {}, 0
        cur[k] = v
        size += nb
    if cur:
        shards.append(cur)
    if len(shards) == 1:
        save_file(shards[0], os.path.join(path, "model.safetensors"), metadata={"format": "pt"})
        return
    index = {"metadata": {"total_size": sum(v.numel() * v.element_size() for _, v in items)},
             "weight_map": {}}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-{len(shards):05d}.safetensors"
        save_file(sh, os.path.join(path, fn), metadata={"format": "pt"})
        for k in sh:
            index["weight_map"][k] = fn
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump(index, f, indent=2)


def load_pretrained_state(path: str, keys: Optional[Iterable[str]] = None) -> Dict[str, torch.Tensor]:
    """Read an HF checkpoint directory (single or sharded safetensors) into a CPU state dict."""
    from safetensors import safe_open
    files = []
    idx = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(idx):
        with open(idx) as f:
            files = sorted(set(json.load(f)["weight_map"].values()))
    else:
        files = ["model.safetensors"]
    want = set(keys) if keys is not None else None
    out = {}
    for fn in files:
        with safe_open(os.path.join(path, fn), framework="pt") as f:
            for k in f.keys():
                if want is None or k in want:
                    out[k] = f.get_tensor(k)
    return out


def save_model(model, path: str) -> None:
    """Save a single-device native model as an HF checkpoint."""
    save_pretrained(path, model.cfg, native_to_hf(model.cfg, dict(model.flat.params)))


def load_model_(model, path: str) -> None:
    hf_to_native_(model.cfg, load_pretrained_state(path), dict(model.flat.params))


def _sha256(path: str) -> str:
    import hashlib
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for blk in iter(lambda: f.read(1 << 20), b""):
            h.update(blk)
    return h.hexdigest()


def save_training_state(path: str, rank: int, shard_state: Dict[str, torch.Tensor],
                        client_state: Dict) -> None:
    """Write this rank's optimizer shard (with a sha256 sidecar) and, on rank 0, the client
    state ``{"step", "completed_steps"}``."""
    d = os.path.join(path, "training_states")
    os.makedirs(d, exist_ok=True)
    f = os.path.join(d, f"optim_rank{rank}.pt")
    tmp = f + ".tmp"
    torch.save({k: v.detach().cpu() for k, v in shard_state.items()}, tmp)
    os.replace(tmp, f)
    with open(f + ".sha256", "w") as fh:
        fh.write(_sha256(f))
    if rank == 0:
        with open(os.path.join(d, "client_state.json"), "w") as f:
            json.dump(client_state, f)
        with open(os.path.join(d, "latest"), "w") as f:
            f.write("train")


def load_training_state(path: str, rank: int):
    """Read this rank's shard (verifying its checksum) and the client state."""
    d = os.path.join(path, "training_states")
    f = os.path.join(d, f"optim_rank{rank}.pt")
    if os.path.exists(f + ".sha256"):
        with open(f + ".sha256") as fh:
            want = fh.read().strip()
        if _sha256(f) != want:
            raise RuntimeError(f"training state {f}: checksum mismatch (corrupted shard)")
    shard = torch.load(f, map_location="cpu")
    with open(os.path.join(d, "client_state.json")) as f:
        client = json.load(f)
    return shard, client
