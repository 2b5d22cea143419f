"""1F1B pipeline x tensor parallel (gloo CPU ranks) equals single-rank training."""
import pytest
import torch

from tests.dist_utils import run_ranks
from tests.test_tp_cpu import _cfg, _full_params


def _batches(cfg, M, B=2, S=40):
    g = torch.Generator().manual_seed(11)
    out = []
    for _ in range(M):
        ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g)
        rl = torch.exp(1.0 + 0.5 * torch.randn(B, S - 1, generator=g))
        out.append((ids, rl))
    return out


def _run(rank, world, tp, pp, M, drop, tmpdir):
    import os

    from centrifuge_b200.models.tp_llama import TPLlamaCore
    from centrifuge_b200.parallel.pipeline import PipelineTrainer, build_groups, stage_layers
    from centrifuge_b200.parallel.zero import ZeroAdamW
    import torch.distributed as dist
    os.environ["CFB_NODE_TRACING_FILE"] = os.path.join(tmpdir, f"d{rank}.txt")
    cfg = _cfg()
    full = _full_params(cfg)
    g = build_groups(tp, pp)
    layers = stage_layers(cfg.num_hidden_layers, pp, g.stage)
    core = TPLlamaCore(cfg, g.tp_group, device="cpu", first=layers.start, last=layers.stop,
                       has_embed=g.stage == 0, has_head=g.stage == pp - 1, dtype=torch.float32)
    core.load_full_(dict(full.flat.params))
    opt = ZeroAdamW(core.flat, group=None, lr=1e-3, grad_clip=1.0, norm_group=dist.group.WORLD,
                    replicated_ranges=core.replicated_ranges(), replication=tp)
    tr = PipelineTrainer(core, opt, g, drop_rate=drop, num_microbatches=M)
    grads = {}
    opt.pre_step_hooks.append(lambda: grads.update(
        {k: v.detach().numpy().copy() for k, v in core.flat.grads.items()}))
    loss = tr.train_step(_batches(cfg, M))
    return {"stage": g.stage, "tp_rank": g.tp_rank, "loss": None if loss is None else float(loss),
            "grads": grads, "norm": float(opt._norm)}


@pytest.mark.parametrize("drop", [0.5, 0.0])
def test_tp2_pp2_matches_single(drop, tmp_path):
    import os

    from centrifuge_b200.models.tp_llama import shard_full_params
    from centrifuge_b200.parallel.zero import ZeroAdamW
    from centrifuge_b200.trainer import Trainer
    from centrifuge_b200.data.synthetic import Batch
    os.environ["CFB_NODE_TRACING_FILE"] = str(tmp_path / "single.txt")
    M = 4
    cfg = _cfg()
    full = _full_params(cfg)
    opt = ZeroAdamW(full.flat, lr=1e-3, grad_clip=1.0)
    want = {}
    opt.pre_step_hooks.append(lambda: want.update(
        {k: v.detach().clone() for k, v in full.flat.grads.items()}))
    tr = Trainer(full, opt, drop_rate=drop, grad_accum=M)
    loss = tr.train_step([Batch(i, r) for i, r in _batches(cfg, M)], to_device=False)
    res = run_ranks(_run, 4, 2, 2, M, drop, str(tmp_path))
    for r in res:
        if r["loss"] is not None:
            assert abs(r["loss"] - float(loss)) < 1e-5
        assert abs(r["norm"] - float(opt._norm)) < 1e-4 * max(1.0, float(opt._norm))
        wp = shard_full_params(cfg, want, 2, r["tp_rank"])
        for name, v in r["grads"].items():
            v = torch.from_numpy(v)
            err = ((v - wp[name]).norm() / (wp[name].norm() + 1e-12)).item()
            assert err < 1e-4, (r["stage"], name, err)


def test_stage_split_balances_head_cost():
    from centrifuge_b200.parallel.pipeline import stage_layers
    # even split without costs (reference stage demo)
    assert [len(stage_layers(22, 4, s)) for s in range(4)] == [6, 6, 5, 5]
    # the last stage also runs the LM head: it gets fewer layers, contiguous and complete
    for L, pp, hc in ((32, 2, 2.2), (32, 4, 5.0), (8, 2, 5.0), (5, 5, 3.0)):
        rs = [stage_layers(L, pp, s, head_cost=hc) for s in range(pp)]
        assert rs[0].start == 0 and rs[-1].stop == L
        assert all(a.stop == b.start and len(a) >= 1 for a, b in zip(rs, rs[1:]))
        costs = [len(r) + (hc if s == pp - 1 else 0.0) for s, r in enumerate(rs)]
        even = [len(stage_layers(L, pp, s)) + (hc if s == pp - 1 else 0.0) for s in range(pp)]
        assert max(costs) <= max(even)
    assert [len(stage_layers(32, 2, s, head_cost=2.2)) for s in range(2)] == [17, 15]
