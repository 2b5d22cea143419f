"""Native Llama (fused single-node backward) against the detached-K/V oracle on CPU."""
import pytest
import torch

from centrifuge_b200.config import tiny_llama_test
from centrifuge_b200.filter import backward_filter
from centrifuge_b200.loss import token_filter_loss
from centrifuge_b200.models.llama import NativeLlamaForCausalLM
from centrifuge_b200.models.reference_llama import ReferenceLlama
from centrifuge_b200.utils.checkpoint import hf_to_native_, native_to_hf


def _models(layers=2):
    cfg = tiny_llama_test(layers=layers, hidden=64, heads=4, kv_heads=2, ffn=128, vocab=256)
    cfg.max_position_embeddings = 256
    torch.manual_seed(0)
    ref = ReferenceLlama(cfg)
    for p in ref.parameters():
        if p.dim() > 1:
            torch.nn.init.normal_(p, std=0.05)
    nat = NativeLlamaForCausalLM(cfg, device="cpu", dtype=torch.float32, init=False)
    hf_to_native_(cfg, ref.state_dict(), dict(nat.flat.params))
    return cfg, ref, nat


def _batch(B, S, vocab, seed=1):
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (B, S), generator=g)
    rl = torch.distributions.LogNormal(1.0, 0.5).sample((B, S - 1))
    return ids, rl


@pytest.mark.parametrize("B,S,drop", [(1, 40, 0.5), (3, 40, 0.5), (2, 72, 0.3), (2, 40, 0.0)])
def test_native_filtered_matches_oracle(B, S, drop, tmp_path, monkeypatch):
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    cfg, ref, nat = _models()
    ids, rl = _batch(B, S, cfg.vocab_size)
    out = nat(ids)
    loss, mask = token_filter_loss(ids, None, torch.ones(B, S, dtype=torch.long), rl.clone(),
                                   "fixed", drop, True, True, per_token_loss=out.token_loss)
    if drop > 0:
        backward_filter(loss, mask)
    loss.backward()
    logits = ref(ids, keep_mask=mask if drop > 0 else None)
    loss_r, mask_r = token_filter_loss(ids, logits, torch.ones(B, S, dtype=torch.long), rl.clone(),
                                       "fixed", drop, True, True)
    assert torch.equal(mask, mask_r)
    assert abs(loss.item() - loss_r.item()) < 1e-4
    loss_r.backward()
    got = native_to_hf(cfg, dict(nat.flat.grads))
    for name, p in ref.named_parameters():
        err = ((got[name] - p.grad).norm() / (p.grad.norm() + 1e-12)).item()
        assert err < 1e-4, (name, err)
