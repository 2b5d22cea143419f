"""Eager-attention HF Llama through the generic graph rewrite, against the reference build.

With ``attn_implementation="eager"`` the attention is plain matmul / softmax nodes, which the
rewrite shrinks like every other node: saved tensors lose their dropped rows in both the query
and the key dimension (the reference's standard build; its ``EAGER_BMM_PROCESS`` variant with
``BmmBackwardFilter`` is off by default, grad_filter/token_filter/csrc/common.h:29).  The oracle
is the reference implementation itself: its ``grad_filter`` extension, built by
``baseline/build_ref.sh``, runs the same model, batch and mask in a subprocess (both libraries
register the ``token_filter`` operator namespace, so they cannot share a process); skipped when
the reference build is absent.  The comparison uses one sequence: for several sequences the
reference shrinks the ``[B*heads, S, S]`` score tensors (batch folded into the first dimension)
with the kept positions of sequence 0 for every sequence (graph_filter.cpp:216-221), while this
rewrite uses each sequence's own positions.  The batched case is checked against the mean of
per-sequence runs instead, which the reference's own semantics give for one sequence.
"""
import glob
import os
import subprocess
import sys

import pytest
import torch

from centrifuge_b200.config import tiny_llama_test
from centrifuge_b200.filter import backward_filter
from centrifuge_b200.filter.probe import build_hf_model
from centrifuge_b200.loss import token_filter_loss

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")
REF_BUILT = bool(glob.glob(os.path.join(REF, "grad_filter", "token_filter", "_C*.so")))


REF_SCRIPT = r"""
import os, sys
repo, ref, path = sys.argv[1], sys.argv[2], sys.argv[3]
sys.path[:] = [p for p in sys.path if os.path.abspath(p or os.getcwd()) != repo]
sys.path.insert(0, ref)
import torch
from transformers import LlamaConfig, LlamaForCausalLM
from grad_filter import token_filter
from model.utils import token_filter_loss
d = torch.load(path)
cfg = LlamaConfig(**d["config"])
cfg._attn_implementation = "eager"
cfg.use_cache = False
model = LlamaForCausalLM(cfg)
model.load_state_dict(d["state"])
model.train()
ids = d["ids"]
am = torch.ones_like(ids)
logits = model(ids, attention_mask=am).logits
loss, mask = token_filter_loss(ids, logits, attention_mask=am, ref_loss=d["ref_loss"].tolist(),
                               dropping_strategy="fixed", drop_rate=0.5, is_left_padding=True,
                               return_mask=True)
token_filter.ops.backward_filter_with_dims(loss, mask, "")
loss.backward()
torch.save({"loss": loss.detach(), "mask": mask,
            "grads": {n: p.grad for n, p in model.named_parameters()}}, path + ".out")
"""


def _case(B, S, seed=1):
    # sizes chosen so that no model dimension equals S, S-1, B*S or B*(S-1): the sequence
    # dimensions are found by value (as in the reference) without a probe batch
    cfg = tiny_llama_test(layers=2, hidden=96, heads=4, kv_heads=2, ffn=160, vocab=256)
    torch.manual_seed(0)
    hf = build_hf_model(cfg.to_hf_dict(), "eager", "cpu", torch.float32)
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g)
    rl = torch.distributions.LogNormal(1.0, 0.5).sample((B, S - 1))
    return cfg, hf, ids, rl


def _filtered_grads(hf, ids, rl):
    B, S = ids.shape
    hf.zero_grad(set_to_none=True)
    logits = hf(input_ids=ids).logits
    loss, mask = token_filter_loss(ids, logits, torch.ones(B, S, dtype=torch.long), rl.clone(),
                                   "fixed", 0.5, True, True)
    backward_filter(loss, mask)
    loss.backward()
    return {n: p.grad.clone() for n, p in hf.named_parameters()}


def test_eager_attention_batch_equals_mean_of_sequences(tmp_path, monkeypatch):
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    cfg, hf, ids, rl = _case(3, 40)
    batched = _filtered_grads(hf, ids, rl)
    (tmp_path / "dims.txt").unlink()
    per = [_filtered_grads(hf, ids[i:i + 1], rl[i:i + 1]) for i in range(3)]
    for name, g in batched.items():
        want = sum(p[name] for p in per) / 3
        err = ((g - want).norm() / (want.norm() + 1e-12)).item()
        assert err < 1e-5, (name, err)


@pytest.mark.skipif(not REF_BUILT, reason="reference build (baseline/_ref) absent")
def test_eager_attention_matches_reference_build(tmp_path, monkeypatch):
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    B, S = 1, 40
    cfg, hf, ids, rl = _case(B, S)
    path = str(tmp_path / "case.pt")
    torch.save({"config": cfg.to_hf_dict(), "state": hf.state_dict(), "ids": ids,
                "ref_loss": rl}, path)
    r = subprocess.run([sys.executable, "-c", REF_SCRIPT, ROOT, REF, path], cwd=str(tmp_path),
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    want = torch.load(path + ".out")

    logits = hf(input_ids=ids).logits
    loss, mask = token_filter_loss(ids, logits, torch.ones(B, S, dtype=torch.long), rl.clone(),
                                   "fixed", 0.5, True, True)
    assert torch.equal(mask, want["mask"])
    assert torch.allclose(loss.detach(), want["loss"], rtol=1e-5)
    backward_filter(loss, mask)
    loss.backward()
    for name, p in hf.named_parameters():
        g_ref = want["grads"][name]
        assert p.grad is not None and g_ref is not None, name
        err = ((p.grad - g_ref).norm() / (g_ref.norm() + 1e-12)).item()
        assert err < 1e-6, (name, err)
