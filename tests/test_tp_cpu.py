"""Tensor + sequence parallel native Llama on gloo CPU ranks equals the single-rank model:
loss, filtered gradients (gathered back to full shape) and one optimizer step."""
import pytest
import torch

from tests.dist_utils import run_ranks


def _cfg():
    from centrifuge_b200.config import tiny_llama_test
    cfg = tiny_llama_test(layers=2, hidden=64, heads=4, kv_heads=2, ffn=128, vocab=256)
    cfg.max_position_embeddings = 128
    return cfg


def _full_params(cfg):
    from centrifuge_b200.models.llama import NativeLlamaForCausalLM
    m = NativeLlamaForCausalLM(cfg, device="cpu", dtype=torch.float32, init=False)
    g = torch.Generator().manual_seed(5)
    for name, p in m.flat.params.items():
        p.copy_(torch.ones_like(p) if p.dim() == 1 else torch.randn(p.shape, generator=g) * 0.05)
    return m


def _batch(cfg, B=2, S=40):
    g = torch.Generator().manual_seed(9)
    ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g)
    rl = torch.exp(1.0 + 0.5 * torch.randn(B, S - 1, generator=g))
    return ids, rl


def _run_tp(rank, world, drop, tmpdir):
    import os

    import torch.distributed as dist

    from centrifuge_b200.filter import backward_filter
    from centrifuge_b200.loss import token_filter_loss
    from centrifuge_b200.models.tp_llama import TPLlamaCore
    os.environ["CFB_NODE_TRACING_FILE"] = os.path.join(tmpdir, f"d{rank}.txt")
    cfg = _cfg()
    full = _full_params(cfg)
    tp = TPLlamaCore(cfg, dist.group.WORLD, device="cpu", dtype=torch.float32)
    tp.load_full_(dict(full.flat.params))
    ids, rl = _batch(cfg)
    out = tp(ids)
    B, S = ids.shape
    loss, mask = token_filter_loss(ids, None, torch.ones(B, S, dtype=torch.long), rl, "fixed",
                                   drop, True, True, per_token_loss=out.token_loss)
    if drop > 0:
        backward_filter(loss, mask)
    loss.backward()
    tp.reduce_replicated_grads()
    return float(loss.detach()), {k: v.detach().numpy().copy() for k, v in tp.flat.grads.items()}


@pytest.mark.parametrize("drop", [0.5, 0.0])
def test_tp2_matches_single(drop, tmp_path):
    from centrifuge_b200.filter import backward_filter
    from centrifuge_b200.loss import token_filter_loss
    from centrifuge_b200.models.tp_llama import shard_full_params
    import os
    os.environ["CFB_NODE_TRACING_FILE"] = str(tmp_path / "single.txt")
    cfg = _cfg()
    full = _full_params(cfg)
    ids, rl = _batch(cfg)
    B, S = ids.shape
    out = full(ids)
    loss, mask = token_filter_loss(ids, None, torch.ones(B, S, dtype=torch.long), rl, "fixed",
                                   drop, True, True, per_token_loss=out.token_loss)
    if drop > 0:
        backward_filter(loss, mask)
    loss.backward()
    want = {k: v.clone() for k, v in full.flat.grads.items()}
    res = run_ranks(_run_tp, 2, drop, str(tmp_path))
    for p, (l, grads) in enumerate(res):
        assert abs(l - float(loss)) < 1e-5
        want_p = shard_full_params(cfg, want, 2, p)
        for name, gp in grads.items():
            gp = torch.from_numpy(gp)
            err = ((gp - want_p[name]).norm() / (want_p[name].norm() + 1e-12)).item()
            assert err < 1e-4, (p, name, err)


class _FakeTP:
    def __init__(self, size, rank):
        self.size, self.rank = size, rank


def test_kept_layout_index_maps():
    """Padded kept-row layout of the filtered TP backward: per-rank counts, the compact <->
    padded maps and the shard-local rows, for several ranks and for one shard (no host read)."""
    from centrifuge_b200.parallel.tensor_parallel import KeptLayout
    T = 32
    rows = torch.tensor([0, 3, 4, 9, 17, 18, 19, 30], dtype=torch.int32)
    P = 4
    lays = [KeptLayout(rows, T, _FakeTP(P, p), "cpu") for p in range(P)]
    assert lays[0].counts == [3, 1, 3, 1] and all(l.C == 3 for l in lays)
    # every compact row lands in its owner's padded slot and maps back
    for l in lays:
        padded = torch.arange(P * l.C)
        assert torch.equal(l.p2c[l.c2p.long()].long(), torch.arange(rows.numel()))
        assert (l.p2c[(padded % l.C) >= torch.tensor(l.counts).repeat_interleave(l.C)] ==
                rows.numel()).all()
    shard = T // P
    for p, l in enumerate(lays):
        mine = rows[(rows // shard) == p] - p * shard
        assert torch.equal(l.local[:l.count], mine)
    one = KeptLayout(rows, T, _FakeTP(1, 0), "cpu")
    assert one.C == one.Tk == one.count == rows.numel() and one.counts == [rows.numel()]
    assert torch.equal(one.local, rows) and torch.equal(one.c2p, torch.arange(8, dtype=torch.int32))
    assert torch.equal(one.p2c, one.c2p) and not one.identity
