"""Cross-tokenizer alignment of reference-model losses onto the target model's tokens.

When the reference model tokenizes a text differently from the model being trained, its
per-token losses must be moved onto the target tokens before the utility selection
(``loss - ref_loss``) can use them.  The reference does this in ``align_ref_target_tokens``
(model/utils.py:548-735) on the decoded token strings (``tokenized_prompts``, stripped of
spaces): it first edits the reference token strings until their concatenation equals the
target's (a windowed character edit distance, model/utils.py:553-680), then walks both token
lists, grouping consecutive tokens until both groups end at the same character, and gives each
target token of a group the group's summed reference loss divided by its number of target
tokens (model/utils.py:689-733).  The first token of each sequence has no loss, so it is
merged into the second before grouping.

This module works on character offsets instead of editing strings:

* token end offsets are cumulative string lengths;
* when the two concatenations differ, reference offsets are mapped into the target string
  through a character alignment (``difflib.SequenceMatcher``: exact inside matching blocks,
  proportional inside edited regions), so every reference token boundary gets a target
  offset;
* the grouping is the reference's greedy walk on those offsets: a group starts with one token
  of each side and grows the side that ends earlier until both end at the same offset.

Target tokens left over when the reference tokens run out get loss 0.0, as in the reference.
"""
from __future__ import annotations

import bisect
import difflib
from typing import List, Sequence


def tokenized_prompts(tokenizer, input_ids: Sequence[Sequence[int]]) -> List[List[str]]:
    """Decoded text of every token, stripped of spaces (model/utils.py:530-537)."""
    return [[tokenizer.decode([int(t)]).strip(" ") for t in ids] for ids in input_ids]


def _ends(tokens: Sequence[str]) -> List[int]:
    out, acc = [], 0
    for t in tokens:
        acc += len(t)
        out.append(acc)
    return out


def _offset_map(src: str, dst: str):
    """Monotone map from character offsets of ``src`` to offsets of ``dst``."""
    if src == dst:
        return lambda o: o
    ops = difflib.SequenceMatcher(None, src, dst, autojunk=False).get_opcodes()
    starts = [op[1] for op in ops]

    def f(o: int) -> int:
        if o >= len(src):
            return len(dst)
        k = max(0, bisect.bisect_right(starts, o) - 1)
        tag, i1, i2, j1, j2 = ops[k]
        if tag == "equal":
            return j1 + (o - i1)
        if i2 == i1:  # pure insertion in dst: src offset sits at its start
            return j1
        return j1 + round((o - i1) * (j2 - j1) / (i2 - i1))

    return f


def align_one(ref_tokens: Sequence[str], target_tokens: Sequence[str],
              ref_loss: Sequence[float]) -> List[float]:
    """Aligned losses of one sequence: one value per target token after the first."""
    if len(target_tokens) < 2:
        return []
    if len(ref_tokens) < 2:
        return [0.0] * (len(target_tokens) - 1)
    ref_str, tgt_str = "".join(ref_tokens), "".join(target_tokens)
    to_tgt = _offset_map(ref_str, tgt_str)
    # tokens 0 and 1 merged: loss token i (i >= 0) ends where token i+1 ends
    r_end = [to_tgt(e) for e in _ends(ref_tokens)[1:]]
    t_end = _ends(target_tokens)[1:]
    losses = list(ref_loss)[:len(r_end)]
    out: List[float] = []
    i = j = 0
    n_r, n_t = min(len(r_end), len(losses)), len(t_end)
    while i < n_r and j < n_t:
        # a group starts with one token of each side
        acc = losses[i]
        j0 = j
        re, te = r_end[i], t_end[j]
        i += 1
        j += 1
        while re != te:
            if re < te:
                if i >= n_r:
                    break
                acc += losses[i]
                re = r_end[i]
                i += 1
            else:
                if j >= n_t:
                    break
                te = t_end[j]
                j += 1
        if re != te:  # one side ran out inside a group: the group is not aligned
            j = j0
            break
        share = acc / (j - j0)
        out.extend([share] * (j - j0))
    out.extend([0.0] * (n_t - len(out)))
    return out


def align_ref_target_tokens(ref_tokens: Sequence[Sequence[str]],
                            target_tokens: Sequence[Sequence[str]],
                            ref_loss: Sequence[Sequence[float]]) -> List[List[float]]:
    """Per sample, the reference losses moved onto the target tokens (``len(target) - 1``
    values each; ``ref_loss[k]`` has ``len(ref_tokens[k]) - 1`` values).  Inputs are not
    modified."""
    return [align_one(r, t, l) for r, t, l in zip(ref_tokens, target_tokens, ref_loss)]
