"""Data-parallel ZeRO-2 on 2+ GPUs: the NVLink peer-memory reducer equals the NCCL baseline."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from centrifuge_b200.config import tiny_llama_test
        from centrifuge_b200.data.synthetic import SyntheticTokenData
        from centrifuge_b200.models.llama import NativeLlamaForCausalLM
        from centrifuge_b200.parallel.symm import SymmReducer
        from centrifuge_b200.parallel.zero import NcclReducer, ZeroAdamW
        from centrifuge_b200.trainer import Trainer
        os.environ["CFB_NODE_TRACING_FILE"] = f"/tmp/cfb_dp_dims_{rank}.txt"
        cfg = tiny_llama_test(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=1024,
                              head_dim=64)
        results = {}
        # (reducer, gradient mode): full local fp32 gradients reduced once per step, or
        # partitioned ZeRO-2 gradients in a ring of bucket slots reduced every micro-batch
        for kind, mode in (("nccl", "full"), ("symm", "full"), ("nccl", "ring"),
                           ("symm", "ring")):
            model = NativeLlamaForCausalLM(cfg, device="cuda", seed=0, pad_to=world,
                                           bucket_numel=1 << 16)
            g = dist.group.WORLD
            red = (SymmReducer.create(model.flat, g, ring=mode == "ring") if kind == "symm"
                   else NcclReducer(g, comm_dtype=torch.float32))
            opt = ZeroAdamW(model.flat, group=g, stage=2, lr=1e-3, bucket_numel=1 << 16,
                            reducer=red, grad_mode=mode)
            assert (model.flat.grad is None) == (mode == "ring")
            tr = Trainer(model, opt, drop_rate=0.5, grad_accum=2, world_size=world)
            data = SyntheticTokenData(cfg.vocab_size, 2, 128, seed=1, rank=rank)
            for _ in range(2):
                tr.train_step([data.sample() for _ in range(2)])
            tr.status.check_now()
            torch.cuda.synchronize()
            if kind == "symm":
                red.check()
                results["kind"] = red.kind
            results[(kind, mode)] = model.flat.data.float().cpu()
        ref = results[("nccl", "full")]
        err = max(((results[k] - ref).norm() / ref.norm()).item()
                  for k in results if k not in ("kind", ("nccl", "full")))
        q.put((rank, err, results.get("kind")))
    finally:
        dist.destroy_process_group()


def test_symm_reducer_matches_nccl():
    import torch.multiprocessing as mp

    from tests.dist_utils import free_port
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = [q.get(timeout=300) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    for rank, err, kind in out:
        assert err < 1e-3, (rank, err, kind)
