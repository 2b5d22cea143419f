"""Cross-tokenizer reference-loss alignment (reference model/utils.py:548-735)."""
import pytest
import torch

from centrifuge_b200.data.align import align_one, align_ref_target_tokens, tokenized_prompts
from centrifuge_b200.data.ref_server import obtain_ref_loss, obtain_ref_loss_cross_tokenizer


def test_same_tokens_keep_losses():
    toks = ["<s>", "a", "bc", "d"]
    assert align_one(toks, toks, [1.0, 2.0, 3.0]) == [1.0, 2.0, 3.0]


def test_grouping_matches_the_reference_walk():
    # Values worked through the reference's loop by hand: tokens 0 and 1 merge ("Thequ" and
    # "The"); "Thequ"+"ick" and "The"+"quick" end together (losses 1+2 over 2 target tokens),
    # then "brown" and "bro"+"wn" (loss 3 over 2 target tokens).
    ref = ["The", "qu", "ick", "brown"]
    tgt = ["Th", "e", "quick", "bro", "wn"]
    assert align_one(ref, tgt, [1.0, 2.0, 3.0]) == [1.5, 1.5, 1.5, 1.5]
    # one reference token spanning three target tokens
    assert align_one(["x", "abc"], ["x", "a", "b", "c"], [6.0]) == [2.0, 2.0, 2.0]
    # three reference tokens summed onto one target token
    assert align_one(["x", "a", "b", "c"], ["x", "abc"], [1.0, 2.0, 4.0]) == [7.0]


def test_mismatched_strings_are_aligned_by_characters():
    # the target text has an extra character: reference boundaries map past it
    out = align_one(["a", "bc", "d"], ["a", "b", "xc", "d"], [4.0, 5.0])
    assert out == [2.0, 2.0, 5.0]
    # the reference text has an extra character
    out = align_one(["a", "b", "yc", "d"], ["a", "bc", "d"], [1.0, 2.0, 3.0])
    assert len(out) == 2 and out[1] == 3.0 and out[0] == pytest.approx(3.0)


def test_trailing_target_text_and_leftover_tokens():
    # target text beyond the reference's: the reference appends it to its last token
    # (model/utils.py:575-577), so that token's loss covers the trailing target tokens
    out = align_one(["a", "b"], ["a", "b", "c", "d"], [5.0])
    assert out == pytest.approx([5.0 / 3] * 3)
    # reference losses that run out before the target tokens: the rest get 0.0
    assert align_one(["a", "b", "c", "d"], ["a", "b", "c", "d"], [5.0]) == [5.0, 0.0, 0.0]
    assert align_one(["a"], ["a", "b"], []) == [0.0]


def test_batch_and_inputs_untouched():
    ref = [["a", "b", "c"], ["x", "yz"]]
    tgt = [["a", "bc"], ["x", "y", "z"]]
    loss = [[1.0, 2.0], [3.0]]
    before = [list(r) for r in ref], [list(t) for t in tgt], [list(l) for l in loss]
    out = align_ref_target_tokens(ref, tgt, loss)
    assert out == [[3.0], [1.5, 1.5]]
    assert (ref, tgt, loss) == before


class _CharTok:
    """Toy tokenizer: one token per character (ids = code points)."""
    add_bos_token = False
    pad_token_id = 0

    def decode(self, ids):
        return "".join(chr(i) for i in ids)

    def batch_decode(self, seqs):
        return [self.decode(s) for s in seqs]

    def __call__(self, texts, **kw):
        return {"input_ids": [[ord(c) for c in t] for t in texts]}


class _PairTok(_CharTok):
    """Toy tokenizer: one token per two characters (ids = 1000 + index in a table)."""

    def __init__(self):
        self.table = []

    def _id(self, piece):
        if piece not in self.table:
            self.table.append(piece)
        return 1000 + self.table.index(piece)

    def decode(self, ids):
        return "".join(self.table[i - 1000] for i in ids)

    def __call__(self, texts, **kw):
        return {"input_ids": [[self._id(t[i:i + 2]) for i in range(0, len(t), 2)] for t in texts]}


class _UnigramLM(torch.nn.Module):
    def __init__(self, vocab=2048):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.logits = torch.nn.Parameter(torch.randn(vocab, generator=g))

    def forward(self, ids):
        return self.logits.expand(ids.shape[0], ids.shape[1], -1)


def test_cross_tokenizer_losses_cover_every_target_token():
    ref_tok, tgt_tok = _CharTok(), _PairTok()
    texts = ["abcdefgh", "hello world!"]
    tgt_ids = tgt_tok(texts)["input_ids"]
    model = _UnigramLM()
    out = obtain_ref_loss_cross_tokenizer(model, ref_tok, tgt_ids, tgt_tok)
    assert [len(o) for o in out] == [len(t) - 1 for t in tgt_ids]
    # every target token after the first covers two reference characters: each gets the sum
    # of the two reference losses of its characters (first group: three characters, two
    # target tokens)
    ref_ids = ref_tok(texts)["input_ids"]
    ref_losses = obtain_ref_loss(model, ref_ids)
    want = align_ref_target_tokens(tokenized_prompts(ref_tok, ref_ids),
                                   tokenized_prompts(tgt_tok, tgt_ids), ref_losses)
    assert out == want
    l0 = ref_losses[0]
    assert out[0][1] == pytest.approx(l0[3] + l0[4])
