"""TP=2 (+SP) on 2 GPUs against the single-GPU native model (bf16 tolerance)."""
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
        from centrifuge_b200.filter import backward_filter
        from centrifuge_b200.loss import token_filter_loss
        from centrifuge_b200.models.llama import NativeLlamaForCausalLM
        from centrifuge_b200.models.tp_llama import TPLlamaCore, shard_full_params
        os.environ["CFB_NODE_TRACING_FILE"] = f"/tmp/cfb_tp_dims_{rank}.txt"
        cfg = tiny_llama_test(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=1024,
                              head_dim=64)
        cfg.max_position_embeddings = 512
        full = NativeLlamaForCausalLM(cfg, device="cuda", seed=0)
        tp = TPLlamaCore(cfg, dist.group.WORLD, device="cuda")
        tp.load_full_(dict(full.flat.params))
        g = torch.Generator().manual_seed(3)
        B, S = 2, 256
        ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g).cuda()
        rl = torch.exp(1.0 + 0.5 * torch.randn(B, S - 1, generator=g)).cuda()
        res = {}
        for name, m in (("full", full), ("tp", tp)):
            out = m(ids)
            loss, mask = token_filter_loss(ids, None, torch.ones(B, S, dtype=torch.long, device="cuda"),
                                           rl, "fixed", 0.5, True, True, per_token_loss=out.token_loss)
            backward_filter(loss, mask)
            loss.backward()
            if name == "tp":
                m.reduce_replicated_grads()
            res[name] = (float(loss.detach()), mask.cpu())
        want = shard_full_params(cfg, {k: v.float() for k, v in full.flat.grads.items()}, world, rank)
        errs = {k: float((tp.flat.grads[k].float() - want[k]).norm() / (want[k].norm() + 1e-12))
                for k in want}
        q.put((rank, res["full"][0], res["tp"][0], bool(torch.equal(res["full"][1], res["tp"][1])),
               max(errs.values())))
    finally:
        dist.destroy_process_group()


def test_tp2_gpu_matches_single_gpu():
    import torch.multiprocessing as mp

    from tests.dist_utils import free_port
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, lf, lt, same_mask, err in out:
        assert abs(lf - lt) < 2e-2 * abs(lf)
        if same_mask:
            assert err < 5e-2, (rank, err)


def _fused_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from centrifuge_b200.config import tiny_llama_test
        from centrifuge_b200.models.tp_llama import TPLlamaCore
        from centrifuge_b200.ops import kernels
        cfg = tiny_llama_test(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=1024,
                              head_dim=64)
        cfg.max_position_embeddings = 512
        tp = TPLlamaCore(cfg, dist.group.WORLD, device="cuda")
        torch.manual_seed(7)
        for v in tp.flat.params.values():
            v.copy_(0.05 * torch.randn_like(v, dtype=torch.float32))
        g = torch.Generator().manual_seed(3)
        B, S = 1, 512  # shards split the sequence: kept rows per rank differ
        ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g).cuda()
        from centrifuge_b200.filter import backward_filter
        from centrifuge_b200.loss import token_filter_loss
        os.environ["CFB_NODE_TRACING_FILE"] = f"/tmp/cfb_tpf_dims_{rank}.txt"
        rl = torch.exp(1.0 + 0.5 * torch.randn(B, S - 1, generator=g)).cuda()
        res = {}
        # dense backward, filtered backward (kept rows per rank differ), and a repeat of both
        for filt, fused in ((False, False), (False, True), (True, False), (True, True),
                            (True, True), (False, True)):
            tp.use_fused_comm = fused
            tp.flat.grad.zero_()
            out = tp(ids).token_loss
            if filt:
                loss, mask = token_filter_loss(ids, None,
                                               torch.ones(B, S, dtype=torch.long, device="cuda"),
                                               rl, "fixed", 0.5, True, True,
                                               per_token_loss=out)
                backward_filter(loss, mask)
            else:
                loss = out.float().mean()
            loss.backward()
            torch.cuda.synchronize()
            res.setdefault((filt, fused), []).append((float(loss.detach()), tp.flat.grad.clone()))
        err_word = kernels().gemm_error_word(rank, True)
        out = []
        for filt in (False, True):
            l0, g0 = res[(filt, False)][0]
            for l1, g1 in res[(filt, True)]:
                out.append((abs(l1 - l0) / abs(l0),
                            float((g1 - g0).norm() / (g0.norm() + 1e-12))))
        q.put((rank, out, err_word, tp._comm.kind))
    finally:
        dist.destroy_process_group()


def test_tp2_fused_collectives_match_nccl():
    """All-gathers fused into RMSNorm (forward and backward) + the consuming GEMM, and
    reduce-scatters fused into the row-parallel (forward) and column-parallel dgrad (backward)
    GEMMs give the same loss and gradients as the NCCL path, dense and with filtering (kept rows
    per rank differ)."""
    import torch.multiprocessing as mp

    from tests.dist_utils import free_port
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_fused_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, rows, err_word, kind in outs:
        assert err_word == 0, (rank, err_word)
        for dl, dg in rows:
            assert dl < 1e-2, (rank, kind, rows)
            assert dg < 3e-2, (rank, kind, rows)


def _pp_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from centrifuge_b200.config import tiny_llama_test
        from centrifuge_b200.models.tp_llama import TPLlamaCore
        from centrifuge_b200.ops import kernels
        from centrifuge_b200.parallel.pipeline import PipelineTrainer, build_groups, stage_layers
        from centrifuge_b200.parallel.zero import ZeroAdamW
        cfg = tiny_llama_test(layers=4, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=1024,
                              head_dim=64)
        cfg.max_position_embeddings = 512
        os.environ["CFB_NODE_TRACING_FILE"] = f"/tmp/cfb_pp_dims_{rank}.txt"
        g = build_groups(2, 2)
        layers = stage_layers(cfg.num_hidden_layers, 2, g.stage)
        core = TPLlamaCore(cfg, g.tp_group, device="cuda", first=layers.start, last=layers.stop,
                           has_embed=g.stage == 0, has_head=g.stage == 1)
        core.comm_sets = 2
        torch.manual_seed(7 + 10 * g.stage + g.tp_rank)
        for v in core.flat.params.values():
            v.copy_(0.05 * torch.randn_like(v, dtype=torch.float32))
        init = core.flat.data.clone()
        gen = torch.Generator().manual_seed(5)
        M, B, S = 4, 1, 512
        batches = [(torch.randint(0, cfg.vocab_size, (B, S), generator=gen).cuda(),
                    torch.exp(1.0 + 0.5 * torch.randn(B, S - 1, generator=gen)).cuda())
                   for _ in range(M)]
        res = []
        for fused in (False, True, True):  # the second fused step reuses the slot sets
            core.flat.data.copy_(init)
            core.use_fused_comm = fused
            opt = ZeroAdamW(core.flat, group=None, lr=1e-4, grad_clip=1.0,
                            norm_group=dist.group.WORLD,
                            replicated_ranges=core.replicated_ranges(), replication=2)
            grads = {}
            opt.pre_step_hooks.append(lambda: grads.update(
                {"all": core.flat.grad.detach().float().clone()}))
            tr = PipelineTrainer(core, opt, g, drop_rate=0.5, num_microbatches=M)
            loss = tr.train_step(batches)
            torch.cuda.synchronize()
            res.append((None if loss is None else float(loss), grads["all"]))
        l0, g0 = res[0]
        out = []
        for l1, g1 in res[1:]:
            dl = 0.0 if l0 is None else abs(l1 - l0) / abs(l0)
            out.append((dl, float((g1 - g0).norm() / (g0.norm() + 1e-12))))
        q.put((rank, out, kernels().gemm_error_word(rank, True),
               core._comm.kind if core._comm is not None else "none"))
    finally:
        dist.destroy_process_group()


def test_tp2_pp2_fused_collectives_match_nccl():
    """Tensor parallel 2 x 1F1B pipeline 2 with the sequence-parallel collectives fused into
    the GEMMs inside every stage (each in-flight micro-batch on its own gather slots) gives the
    NCCL pipeline's loss and gradients, over two steps."""
    import torch.multiprocessing as mp

    from tests.dist_utils import free_port
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_pp_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=300) for _ in range(4)]
    for p in ps:
        p.join(timeout=60)
    for rank, rows, err_word, kind in outs:
        assert err_word == 0, (rank, err_word)
        for dl, dg in rows:
            assert dl < 1e-2, (rank, kind, rows)
            assert dg < 3e-2, (rank, kind, rows)


def _ce_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        from centrifuge_b200.ops import kernels
        from centrifuge_b200.parallel.tensor_parallel import TPGroup
        from centrifuge_b200.parallel.tp_fused import VocabParallelCE
        tp = TPGroup(dist.group.WORLD)
        V = 1000 * world
        x = VocabParallelCE(tp, 512, "cuda")
        errs = []
        for call, T in enumerate((512, 300, 512, 77)):  # slots alternate, rows vary
            g = torch.Generator(device="cuda").manual_seed(100 + call)
            logits = (4 * torch.randn(T, V, generator=g, device="cuda")).bfloat16()
            labels = torch.randint(0, V, (T,), generator=g, device="cuda")
            labels[::7] = -100
            shard = logits[:, rank * 1000:(rank + 1) * 1000].contiguous()
            loss, lse = x(shard, labels, rank * 1000)
            lf = logits.float()
            want_lse = torch.logsumexp(lf, -1)
            want = torch.nn.functional.cross_entropy(lf, labels.clamp(min=0), reduction="none")
            want = torch.where(labels >= 0, want, torch.zeros_like(want))
            torch.cuda.synchronize()
            errs.append(max(float((loss - want).abs().max()), float((lse - want_lse).abs().max())))
        q.put((rank, errs, kernels().gemm_error_word(rank, True)))
    finally:
        dist.destroy_process_group()


def test_tp2_vocab_parallel_ce_exchange():
    """Vocabulary-parallel cross entropy with the row statistics exchanged over NVLink equals the
    fp32 cross entropy of the full logits, over calls that alternate the buffer slots."""
    import torch.multiprocessing as mp

    from tests.dist_utils import free_port
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    ps = [ctx.Process(target=_ce_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    outs = [q.get(timeout=300) for _ in range(2)]
    for p in ps:
        p.join(timeout=60)
    for rank, errs, err_word in outs:
        assert err_word == 0, (rank, err_word)
        assert max(errs) < 2e-3, (rank, errs)
