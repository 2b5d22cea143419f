"""Token selection and filtered loss against a direct per-row restatement of the reference
loop (model/utils.py:398-424), plus property tests."""
import pytest
import torch

from centrifuge_b200.loss import (align_drop_rate, keep_count, loss_average, num_dropped,
                                  token_dropping_mask, token_filter_loss)


def _reference_fixed(loss, ref_loss, mask, drop_rate, left=True):
    mask = mask.clone()
    diff = loss - ref_loss
    seq_len = loss.shape[1]
    filter_len = int(seq_len * drop_rate)
    if filter_len % 8 != 0:
        filter_len += 8 - filter_len % 8
        drop_rate = filter_len / seq_len + 0.5 / seq_len
    for i in range(loss.shape[0]):
        n = int(mask[i].sum().item()) - 1
        start = int(mask.shape[1] - n - 1) if left else 1
        end = (mask.shape[1] - 1) if left else int(n + 1)
        k = int(drop_rate * n)
        _, idx = torch.topk(diff[i][start:end], k, largest=False)
        mask[i].scatter_(0, idx + start, 0)
    return mask


@pytest.mark.parametrize("S,drop", [(224, 0.5), (2048, 0.5), (4096, 0.3), (4096, 0.7),
                                    (100, 0.2), (17, 0.6)])
def test_fixed_matches_reference_loop(S, drop):
    g = torch.Generator().manual_seed(S)
    B = 3
    loss = torch.rand(B, S - 1, generator=g) * 5
    ref = torch.distributions.LogNormal(1.0, 0.5).sample((B, S - 1))
    m = torch.ones(B, S, dtype=torch.long)
    want = _reference_fixed(loss, ref, m, drop)
    got = token_dropping_mask(loss, ref, m.clone(), "fixed", drop, True)
    assert torch.equal(got, want)
    # properties: S_keep = S - round_up_8(int(drop*(S-1))), last position kept
    k = num_dropped(S, drop)
    assert k % 8 == 0 or k == int(align_drop_rate(drop, S - 1) * (S - 1))
    assert (got.sum(1) == S - k).all() and (got[:, -1] == 1).all()
    assert keep_count(S, drop) == S - k


def test_left_padded_rows():
    g = torch.Generator().manual_seed(0)
    B, S = 2, 40
    loss = torch.rand(B, S - 1, generator=g)
    ref = torch.rand(B, S - 1, generator=g)
    m = torch.ones(B, S, dtype=torch.long)
    m[0, :10] = 0  # left padding on row 0
    want = _reference_fixed(loss, ref, m, 0.5)
    got = token_dropping_mask(loss, ref, m.clone(), "fixed", 0.5, True)
    assert torch.equal(got, want)


@pytest.mark.parametrize("strategy", ["positive", "self", "less_ref", "peaking"])
def test_other_strategies_run_and_drop(strategy, tmp_path):
    g = torch.Generator().manual_seed(1)
    B, S = 2, 64
    loss = torch.rand(B, S - 1, generator=g) * 3
    ref = torch.rand(B, S - 1, generator=g) * 3
    m = torch.ones(B, S, dtype=torch.long)
    kw = {}
    out = token_dropping_mask(loss, ref, m, strategy, 0.4, True, **kw)
    assert out.sum() < B * S and out[:, -1].eq(1).all()


def test_dynamic_not_implemented():
    with pytest.raises(NotImplementedError):
        token_dropping_mask(torch.rand(1, 7), torch.rand(1, 7), torch.ones(1, 8, dtype=torch.long),
                            "dynamic", 0.5, True)


def test_token_filter_loss_is_masked_mean():
    g = torch.Generator().manual_seed(2)
    B, S, V = 2, 24, 50
    ids = torch.randint(0, V, (B, S), generator=g)
    logits = torch.randn(B, S, V, generator=g)
    ref = [[0.1] * (S - 1), [0.2] * (S - 5)]  # ragged: left-padded with zeros
    loss, mask = token_filter_loss(ids, logits, torch.ones(B, S, dtype=torch.long), ref, "fixed",
                                   0.5, True, True)
    per_tok = torch.nn.functional.cross_entropy(logits[:, :-1].reshape(-1, V), ids[:, 1:].reshape(-1),
                                                reduction="none").view(B, S - 1)
    lm = mask[:, :-1].float()
    want = ((per_tok * lm).sum(1) / lm.sum(1)).mean()
    assert torch.allclose(loss, want)
    assert torch.allclose(loss_average(per_tok, mask, is_left_padding=True), want)
