"""ZeRO-1/2 data parallel on gloo CPU ranks equals single-rank training on the same batches."""
import pytest
import torch

from tests.dist_utils import run_ranks


def _setup(world, seed=0, bucket_numel=1 << 26):
    from centrifuge_b200.config import tiny_llama_test
    from centrifuge_b200.models.llama import NativeLlamaForCausalLM
    cfg = tiny_llama_test(layers=2, hidden=64, heads=4, kv_heads=2, ffn=128, vocab=256)
    cfg.max_position_embeddings = 128
    torch.manual_seed(seed)
    model = NativeLlamaForCausalLM(cfg, device="cpu", dtype=torch.float32, init=False,
                                   pad_to=world, bucket_numel=bucket_numel)
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


def _train(rank, world, stage, ga, steps, tmpdir, every=False, mode="full"):
    import os

    import torch.distributed as dist

    from centrifuge_b200.parallel.zero import NcclReducer, ZeroAdamW
    from centrifuge_b200.trainer import Trainer
    os.environ["CFB_NODE_TRACING_FILE"] = os.path.join(tmpdir, f"dims{rank}.txt")
    # small buckets: several buckets per layer, so the gradient ring cycles within a step
    cfg, model = _setup(world, bucket_numel=4096)
    group = dist.group.WORLD if world > 1 else None
    red = NcclReducer(group, comm_dtype=torch.float32) if world > 1 else None
    opt = ZeroAdamW(model.flat, group=group, stage=stage, lr=1e-3, grad_clip=1.0,
                    bucket_numel=4096, reducer=red, reduce_every_micro=every,
                    grad_mode=mode if world > 1 else "full")
    if mode == "ring" and world > 1:
        assert model.flat.grad is None and opt.ring is not None
        assert len(opt.buckets) > opt.ring.R  # slots are reused within a micro-batch
    tr = Trainer(model, opt, drop_rate=0.5, grad_accum=ga, world_size=world)
    allb = _batches(cfg, steps * ga * world)
    for s in range(steps):
        chunk = allb[s * ga * world:(s + 1) * ga * world]
        mine = chunk[rank * ga:(rank + 1) * ga]
        tr.train_step(mine, to_device=False)
    params = {n: p.detach().numpy().copy() for n, p in model.flat.params.items()}
    return params, float(opt._norm.item()), opt.grad_memory_bytes()


@pytest.mark.parametrize("stage,every,mode", [(1, False, "full"), (2, False, "full"),
                                              (2, True, "full"), (2, False, "ring")])
def test_zero_matches_single_rank(stage, every, mode, tmp_path):
    """Stage 2: full local gradients reduced in the last micro-batch's backward (default) or in
    every one, or partitioned gradients in a ring of bucket slots reduced in every micro-batch."""
    world, ga, steps = 2, 2, 2
    multi = run_ranks(_train, world, stage, ga, steps, str(tmp_path), every, mode)
    single = _train(0, 1, stage, ga * world, steps, str(tmp_path))
    for r in range(world):
        params, norm, gbytes = multi[r]
        for name, ref in single[0].items():
            assert torch.allclose(torch.from_numpy(params[name]), torch.from_numpy(ref),
                                  atol=1e-5), (stage, mode, r, name)
        assert abs(norm - single[1]) < 1e-4 * max(1.0, single[1])


@pytest.mark.parametrize("world", [2, 8])
def test_ring_gradient_memory_at_tinyllama_scale(world):
    """Bucket layout and gradient memory of partitioned ZeRO-2 for TinyLlama-1.1B (meta
    tensors): parameters never straddle buckets, buckets split into aligned rank chunks, and the
    ring plus the fp32 shard take far less than a full fp32 gradient buffer."""
    from centrifuge_b200.config import get_model_config
    from centrifuge_b200.models.flat import ALIGN_ELEMS, FlatParams
    from centrifuge_b200.models.llama import param_specs
    from centrifuge_b200.parallel.zero import _buckets_per_unit
    cfg = get_model_config("TinyLlama-1.1B")
    specs = param_specs(cfg, range(cfg.num_hidden_layers), True, True)
    flat = FlatParams(specs, "meta", pad_to=world, bucket_numel=1 << 26)
    bounds = flat.bucket_bounds
    assert bounds[0][0] == 0 and bounds[-1][1] == flat.numel
    for (lo, hi), (lo2, _) in zip(bounds, bounds[1:]):
        assert hi == lo2 and (hi - lo) % (world * ALIGN_ELEMS) == 0
    for name, shape in flat.specs.items():
        lo, hi = flat.range_of(name)
        assert any(blo <= lo and hi <= bhi for blo, bhi in bounds), name
    slots = max(4, _buckets_per_unit(flat) + 1)
    ring = slots * max(hi - lo for lo, hi in bounds) * 4
    shard = flat.numel // world * 4
    full = flat.numel * 4
    # TinyLlama: 24 buckets of <= 65.5M elements, 4 slots = 1.05 GB against 4.4 GB
    assert ring < 0.25 * full and ring + shard < full, (ring, shard, full)


@pytest.mark.parametrize("mode", ["ring", "full"])
def test_data_parallel_training_is_deterministic(mode, tmp_path):
    """Distributed determinism: two identical 2-rank ZeRO-2 runs give bit-identical parameters,
    and after every step's parameter all-gather all ranks hold the same bits."""
    world, ga, steps = 2, 2, 2
    a = run_ranks(_train, world, 2, ga, steps, str(tmp_path / "a"), False, mode)
    b = run_ranks(_train, world, 2, ga, steps, str(tmp_path / "b"), False, mode)
    for name in a[0][0]:
        for r in range(world):
            assert (a[r][0][name] == b[r][0][name]).all(), (mode, r, name)
        assert (a[0][0][name] == a[1][0][name]).all(), (mode, name)
    assert a[0][1] == b[0][1]
