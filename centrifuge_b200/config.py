"""Model and workload configurations.

The model configs describe the Llama-family architectures that the reference trains through
HuggingFace ``AutoModelForCausalLM`` (train.py:428) and through its Megatron TP model
(model/megatronlm.py:9-43).  The workload configs are the benchmark shapes the framework is
measured on: TinyLlama-1.1B data parallel (ZeRO-2), Llama-3-8B tensor/sequence parallel, and
Llama-3-8B TP x PP with a 1F1B schedule.
"""
from __future__ import annotations

import dataclasses
import json
from dataclasses import dataclass, field
from typing import Optional


@dataclass
class LlamaConfig:
    """Decoder-only Llama architecture (RMSNorm, RoPE, GQA attention, SwiGLU FFN)."""

    vocab_size: int = 32000
    hidden_size: int = 2048
    intermediate_size: int = 5632
    num_hidden_layers: int = 22
    num_attention_heads: int = 32
    num_key_value_heads: int = 4
    head_dim: Optional[int] = None
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    max_position_embeddings: int = 2048
    tie_word_embeddings: bool = False
    initializer_range: float = 0.02
    bos_token_id: int = 1
    eos_token_id: int = 2
    name: str = "llama"

    def __post_init__(self):
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_attention_heads
        assert self.num_attention_heads % self.num_key_value_heads == 0

    @property
    def q_size(self) -> int:
        return self.num_attention_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    def num_params(self) -> int:
        h, f, v = self.hidden_size, self.intermediate_size, self.vocab_size
        per_layer = h * self.qkv_size + self.q_size * h + 3 * h * f + 2 * h
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return self.num_hidden_layers * per_layer + emb + h

    def to_hf_dict(self) -> dict:
        """HuggingFace ``config.json`` contents for ``LlamaForCausalLM``."""
        return {
            "architectures": ["LlamaForCausalLM"],
            "model_type": "llama",
            "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size,
            "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads,
            "head_dim": self.head_dim,
            "rms_norm_eps": self.rms_norm_eps,
            "rope_theta": self.rope_theta,
            "max_position_embeddings": self.max_position_embeddings,
            "tie_word_embeddings": self.tie_word_embeddings,
            "hidden_act": "silu",
            "attention_bias": False,
            "mlp_bias": False,
            "initializer_range": self.initializer_range,
            "bos_token_id": self.bos_token_id,
            "eos_token_id": self.eos_token_id,
            "torch_dtype": "bfloat16",
        }

    @classmethod
    def from_hf_dict(cls, d: dict) -> "LlamaConfig":
        names = {f.name for f in dataclasses.fields(cls)}
        kw = {k: v for k, v in d.items() if k in names}
        return cls(**kw)

    def save(self, path: str) -> None:
        with open(path, "w") as f:
            json.dump(self.to_hf_dict(), f, indent=2)

    @classmethod
    def load(cls, path: str) -> "LlamaConfig":
        with open(path) as f:
            return cls.from_hf_dict(json.load(f))


def tinyllama_1b() -> LlamaConfig:
    """TinyLlama-1.1B: 22 layers, hidden 2048, 32 heads / 4 KV heads, FFN 5632, vocab 32000."""
    return LlamaConfig(vocab_size=32000, hidden_size=2048, intermediate_size=5632,
                       num_hidden_layers=22, num_attention_heads=32, num_key_value_heads=4,
                       rms_norm_eps=1e-5, rope_theta=10000.0, max_position_embeddings=2048,
                       name="TinyLlama-1.1B")


def llama3_8b() -> LlamaConfig:
    """Llama-3-8B: 32 layers, hidden 4096, 32 heads / 8 KV heads, FFN 14336, vocab 128256."""
    return LlamaConfig(vocab_size=128256, hidden_size=4096, intermediate_size=14336,
                       num_hidden_layers=32, num_attention_heads=32, num_key_value_heads=8,
                       rms_norm_eps=1e-5, rope_theta=500000.0, max_position_embeddings=8192,
                       bos_token_id=128000, eos_token_id=128001, name="Llama-3-8B")


def tiny_llama_test(layers: int = 2, hidden: int = 128, heads: int = 4, kv_heads: int = 2,
                    ffn: int = 256, vocab: int = 512, head_dim: Optional[int] = None) -> LlamaConfig:
    """A small Llama used by unit tests (same architecture, tiny sizes)."""
    return LlamaConfig(vocab_size=vocab, hidden_size=hidden, intermediate_size=ffn,
                       num_hidden_layers=layers, num_attention_heads=heads,
                       num_key_value_heads=kv_heads, head_dim=head_dim, name="tiny-llama")


MODEL_CONFIGS = {
    "tinyllama-1.1b": tinyllama_1b,
    "TinyLlama/TinyLlama_v1.1": tinyllama_1b,
    "TinyLlama-1.1B": tinyllama_1b,
    "llama-3-8b": llama3_8b,
    "meta-llama/Meta-Llama-3-8B": llama3_8b,
    "Llama-3-8B": llama3_8b,
    "tiny": tiny_llama_test,
}


def get_model_config(name: str) -> LlamaConfig:
    """Resolve a model name or a directory holding ``config.json``."""
    import os
    if name in MODEL_CONFIGS:
        return MODEL_CONFIGS[name]()
    p = os.path.join(name, "config.json")
    if os.path.exists(p):
        return LlamaConfig.load(p)
    raise KeyError(f"unknown model {name!r}; known: {sorted(MODEL_CONFIGS)}")


@dataclass
class TrainConfig:
    """One training workload.  ``parallelism`` is e.g. ``dp8``, ``tp8``, ``tp4pp2``."""

    model: str = "tinyllama-1.1b"
    seq_len: int = 2048
    micro_batch: int = 8
    grad_accum: int = 4
    drop_rate: float = 0.5
    dropping_strategy: str = "fixed"
    zero_stage: int = 2
    tp: int = 1
    pp: int = 1
    sequence_parallel: bool = False
    num_microbatches: int = 1
    lr: float = 1e-4
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    weight_decay: float = 0.0
    grad_clip: float = 1.0
    seed: int = 4321
    ref_loss_mu: float = 1.0
    ref_loss_sigma: float = 0.5
    extra: dict = field(default_factory=dict)


# Benchmark workloads: synthetic uniform token ids, LogNormal(1.0, 0.5) per-token ref_loss,
# random-init weights.
WORKLOADS = {
    "tinyllama_zero2": TrainConfig(model="tinyllama-1.1b", seq_len=2048, micro_batch=8,
                                   grad_accum=4, drop_rate=0.5, zero_stage=2, lr=1e-4,
                                   betas=(0.9, 0.95)),
    "llama3_8b_tp8_sp": TrainConfig(model="llama-3-8b", seq_len=4096, micro_batch=1,
                                    grad_accum=32, drop_rate=0.5, zero_stage=1, tp=8,
                                    sequence_parallel=True),
    "llama3_8b_tp4_pp2": TrainConfig(model="llama-3-8b", seq_len=4096, micro_batch=2,
                                     grad_accum=1, num_microbatches=8, drop_rate=0.5,
                                     zero_stage=1, tp=4, pp=2, sequence_parallel=False),
}
