"""CPU correctness config: the full TinyLlama-1.1B architecture in fp32, one sequence of 224.

22 layers, hidden 2048, 32 heads / 4 K/V heads (head_dim 64), SwiGLU FFN 5632, RMSNorm eps 1e-5,
RoPE theta 10000, vocab 32000, random-init weights; token ids uniform over the vocabulary,
per-token ref_loss ~ LogNormal(1.0, 0.5); the top 50% of tokens by (token loss - ref_loss) are
kept.  Checked:

* the native model's filtered backward and the graph rewrite of a HuggingFace Llama both equal
  the filtered-gradient oracle (K/V of dropped positions detached, mask-weighted loss);
* the oracle's lm_head, final-norm, last-layer MLP, o_proj and q_proj gradients equal those of
  an unfiltered backward of the same masked loss (those parameters see dropped positions only
  through zero-weighted loss terms).
"""
import gc

import pytest
import torch

from centrifuge_b200.config import get_model_config
from centrifuge_b200.filter import backward_filter
from centrifuge_b200.filter.probe import build_hf_model
from centrifuge_b200.loss import token_filter_loss
from centrifuge_b200.models.llama import NativeLlamaForCausalLM
from centrifuge_b200.models.reference_llama import ReferenceLlama
from centrifuge_b200.utils.checkpoint import hf_to_native_, native_to_hf

pytestmark = pytest.mark.slow

B, S = 1, 224


def _rel(a, b):
    return ((a - b).norm() / (b.norm() + 1e-12)).item()


@pytest.fixture(scope="module")
def oracle():
    torch.set_num_threads(max(1, torch.get_num_threads()))
    cfg = get_model_config("TinyLlama-1.1B")
    torch.manual_seed(0)
    ref = ReferenceLlama(cfg)
    with torch.no_grad():
        for p in ref.parameters():
            if p.dim() > 1:
                p.normal_(0.0, 0.02)
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g)
    rl = torch.exp(1.0 + 0.5 * torch.randn(B, S - 1, generator=g))
    # mask from the plain forward, then the filtered oracle backward
    with torch.no_grad():
        _, mask = token_filter_loss(ids, ref(ids), torch.ones(B, S, dtype=torch.long),
                                    rl.clone(), "fixed", 0.5, True, True)
    loss, mask_r = token_filter_loss(ids, ref(ids, keep_mask=mask),
                                     torch.ones(B, S, dtype=torch.long), rl.clone(), "fixed",
                                     0.5, True, True)
    assert torch.equal(mask, mask_r)
    loss.backward()
    grads = {n: p.grad.detach().clone() for n, p in ref.named_parameters()}
    state = {k: v.detach().clone() for k, v in ref.state_dict().items()}
    out = {"cfg": cfg, "ids": ids, "rl": rl, "mask": mask, "loss": loss.item(),
           "grads": grads, "state": state, "model": ref}
    yield out
    out.clear()
    gc.collect()


def test_config0_mask_keeps_half():
    # covered by the fixture's assertions; the selection keeps S - round_up_8(int(0.5*(S-1)))
    from centrifuge_b200.loss import keep_count
    assert keep_count(S, 0.5) == S - 112


def test_config0_unfiltered_masked_backward_cross_check(oracle):
    ref = oracle["model"]
    ref.zero_grad(set_to_none=True)
    ids, mask = oracle["ids"], oracle["mask"]
    logits = ref(ids)  # no detach: the dense backward of the masked loss
    loss = token_filter_loss(ids, logits, mask.clone(), None, None, None, True)
    assert abs(loss.item() - oracle["loss"]) < 1e-4 * abs(oracle["loss"])
    loss.backward()
    last = oracle["cfg"].num_hidden_layers - 1
    names = ["lm_head.weight", "model.norm.weight",
             f"model.layers.{last}.mlp.gate_proj.weight", f"model.layers.{last}.mlp.up_proj.weight",
             f"model.layers.{last}.mlp.down_proj.weight",
             f"model.layers.{last}.post_attention_layernorm.weight",
             f"model.layers.{last}.self_attn.o_proj.weight",
             f"model.layers.{last}.self_attn.q_proj.weight"]
    got = dict(ref.named_parameters())
    for n in names:
        assert _rel(got[n].grad, oracle["grads"][n]) < 1e-4, n
    # and the K/V projections of the last layer do differ: dropped positions' K/V are detached
    kname = f"model.layers.{last}.self_attn.k_proj.weight"
    assert _rel(got[kname].grad, oracle["grads"][kname]) > 1e-3
    ref.zero_grad(set_to_none=True)


def test_config0_native_filtered_matches_oracle(oracle, tmp_path, monkeypatch):
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    cfg = oracle["cfg"]
    nat = NativeLlamaForCausalLM(cfg, device="cpu", dtype=torch.float32, init=False)
    hf_to_native_(cfg, oracle["state"], dict(nat.flat.params))
    ids = oracle["ids"]
    out = nat(ids)
    loss, mask = token_filter_loss(ids, None, torch.ones(B, S, dtype=torch.long),
                                   oracle["rl"].clone(), "fixed", 0.5, True, True,
                                   per_token_loss=out.token_loss)
    assert torch.equal(mask, oracle["mask"])
    backward_filter(loss, mask)
    loss.backward()
    got = native_to_hf(cfg, dict(nat.flat.grads))
    worst = max((_rel(got[n], g), n) for n, g in oracle["grads"].items())
    assert worst[0] < 2e-4, worst
    del nat, got, out
    gc.collect()


def test_config0_hf_rewrite_matches_oracle(oracle, tmp_path, monkeypatch):
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    cfg = oracle["cfg"]
    hf = build_hf_model(cfg.to_hf_dict(), "sdpa", "cpu", torch.float32)
    hf.load_state_dict(oracle["state"], strict=True)
    ids = oracle["ids"]
    logits = hf(input_ids=ids).logits
    loss, mask = token_filter_loss(ids, logits, torch.ones(B, S, dtype=torch.long),
                                   oracle["rl"].clone(), "fixed", 0.5, True, True)
    assert torch.equal(mask, oracle["mask"])
    backward_filter(loss, mask)
    loss.backward()
    got = dict(hf.named_parameters())
    worst = max((_rel(got[n].grad, g), n) for n, g in oracle["grads"].items())
    assert worst[0] < 2e-4, worst
    del hf, got
    gc.collect()
