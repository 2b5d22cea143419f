"""ZeRO-1/2 data parallel on gloo CPU ranks equals single-rank training on the same batches."""
import pytest
import torch

from tests.dist_utils import run_ranks


def _setup(world, seed=0):
    from centrifuge_b200.config import tiny_llama_test
    from centrifuge_b200.models.llama import NativeLlamaForCausalLM
    cfg = tiny_llama_test(layers=2, hidden=64, heads=4, kv_heads=2, ffn=128, vocab=256)
    cfg.max_position_embeddings = 128
    torch.manual_seed(seed)
    model = NativeLlamaForCausalLM(cfg, device="cpu", dtype=torch.float32, init=False,
                                   pad_to=world)
    g = torch.Generator().manual_seed(123)
    for name, p in model.flat.params.items():
        if p.dim() == 1:
            p.fill_(1.0)
        else:
            p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    return cfg, model


def _batches(cfg, n, B=2, S=40):
    from centrifuge_b200.data.synthetic import Batch
    g = torch.Generator().manual_seed(7)
    out = []
    for _ in range(n):
        ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g)
        rl = torch.exp(1.0 + 0.5 * torch.randn(B, S - 1, generator=g))
        out.append(Batch(ids, rl))
    return out


def _train(rank, world, stage, ga, steps, tmpdir, every=False):
    import os

    import torch.distributed as dist

    from centrifuge_b200.parallel.zero import NcclReducer, ZeroAdamW
    from centrifuge_b200.trainer import Trainer
    os.environ["CFB_NODE_TRACING_FILE"] = os.path.join(tmpdir, f"dims{rank}.txt")
    cfg, model = _setup(world)
    group = dist.group.WORLD if world > 1 else None
    red = NcclReducer(group, comm_dtype=torch.float32) if world > 1 else None
    opt = ZeroAdamW(model.flat, group=group, stage=stage, lr=1e-3, grad_clip=1.0,
                    bucket_numel=4096, reducer=red, reduce_every_micro=every)
    tr = Trainer(model, opt, drop_rate=0.5, grad_accum=ga, world_size=world)
    allb = _batches(cfg, steps * ga * world)
    for s in range(steps):
        chunk = allb[s * ga * world:(s + 1) * ga * world]
        mine = chunk[rank * ga:(rank + 1) * ga]
        tr.train_step(mine, to_device=False)
    return model.flat.data.numpy().copy(), float(opt._norm.item())


@pytest.mark.parametrize("stage,every", [(1, False), (2, False), (2, True)])
def test_zero_matches_single_rank(stage, every, tmp_path):
    """Stage 2 reduces in the last micro-batch's backward (default) or in every one."""
    world, ga, steps = 2, 2, 2
    multi = run_ranks(_train, world, stage, ga, steps, str(tmp_path), every)
    single = _train(0, 1, stage, ga * world, steps, str(tmp_path))
    for r in range(world):
        p, norm = multi[r]
        p, ref = torch.from_numpy(p), torch.from_numpy(single[0])
        n = ref.numel()
        assert torch.allclose(p[:n], ref[:n], atol=1e-5), (stage, r)
        assert abs(norm - single[1]) < 1e-4 * max(1.0, single[1])
