"""Generic graph rewrite on a HuggingFace Llama (CPU, fp32) against the detached-K/V oracle."""
import os

import pytest
import torch

from centrifuge_b200.config import tiny_llama_test
from centrifuge_b200.filter import backward_filter, backward_filter_with_dims, collect_node_names
from centrifuge_b200.filter.probe import build_hf_model
from centrifuge_b200.loss import token_filter_loss
from centrifuge_b200.models.reference_llama import ReferenceLlama


def _pair(seed=0, layers=2):
    cfg = tiny_llama_test(layers=layers, hidden=64, heads=4, kv_heads=2, ffn=128, vocab=256)
    torch.manual_seed(seed)
    hf = build_hf_model(cfg.to_hf_dict(), "sdpa", "cpu", torch.float32)
    ref = ReferenceLlama(cfg)
    ref.load_state_dict(hf.state_dict(), strict=True)
    return cfg, hf, ref


def _batch(B, S, vocab, seed=1):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (B, S), generator=g)
    ref_loss = torch.distributions.LogNormal(1.0, 0.5).sample((B, S - 1))
    return ids, ref_loss


@pytest.mark.parametrize("B,S", [(1, 40), (3, 40), (2, 72)])
def test_hf_filtered_grads_match_oracle(B, S, tmp_path, monkeypatch):
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    cfg, hf, ref = _pair()
    ids, rl = _batch(B, S, cfg.vocab_size)
    mask = torch.ones(B, S, dtype=torch.long)
    logits = hf(input_ids=ids).logits
    loss, mask = token_filter_loss(ids, logits, mask, rl.clone(), "fixed", 0.5, True, True)
    backward_filter(loss, mask)
    loss.backward()
    # oracle: same mask, K/V of dropped positions detached, masked loss
    logits_r = ref(ids, keep_mask=mask)
    loss_r, mask_r = token_filter_loss(ids, logits_r, torch.ones(B, S, dtype=torch.long),
                                       rl.clone(), "fixed", 0.5, True, True)
    assert torch.equal(mask, mask_r)
    loss_r.backward()
    hp = dict(hf.named_parameters())
    for name, p in ref.named_parameters():
        g1, g2 = hp[name].grad, p.grad
        assert g1 is not None, name
        err = (g1 - g2).norm() / (g2.norm() + 1e-12)
        assert err < 1e-4, (name, err.item())


def test_dims_record_and_replay(tmp_path, monkeypatch):
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    cfg, hf, ref = _pair(layers=1)
    # record on a probe batch (S=24), replay on a longer one (S=48)
    ids, rl = _batch(1, 24, cfg.vocab_size)
    loss, mask = token_filter_loss(ids, hf(input_ids=ids).logits, None, rl, "fixed", 0.5, True, True)
    dims = backward_filter_with_dims(loss, mask, "")
    assert "---" in dims and "FilteredAttentionBackward" not in dims
    loss.backward()
    hf.zero_grad()
    ids, rl = _batch(1, 48, cfg.vocab_size, seed=3)
    loss, mask = token_filter_loss(ids, hf(input_ids=ids).logits, None, rl, "fixed", 0.5, True, True)
    out = backward_filter_with_dims(loss, mask, dims)
    assert out == dims
    loss.backward()
    logits_r = ref(ids, keep_mask=mask)
    loss_r = token_filter_loss(ids, logits_r, mask.clone(), None, None, None, True)
    loss_r.backward()
    hp = dict(hf.named_parameters())
    for name, p in ref.named_parameters():
        err = (hp[name].grad - p.grad).norm() / (p.grad.norm() + 1e-12)
        assert err < 1e-4, (name, err.item())


def test_collect_node_names():
    cfg, hf, _ = _pair(layers=1)
    ids, rl = _batch(1, 16, cfg.vocab_size)
    loss, _ = token_filter_loss(ids, hf(input_ids=ids).logits, None, rl, "fixed", 0.5, True, True)
    names = collect_node_names(loss)
    assert "ScaledDotProductFlashAttentionForCpuBackward0" in names
    assert "torch::autograd::AccumulateGrad" in names
