"""Device-side failure reporting: bounded waits that run out, and what the step does after.

The failure is made without faulting or hanging the GPU: a wait on a flag that nothing raises,
with the peer wait limit shortened to 5 ms at run time, records its error code and returns.  The
test then checks that the kernels after it skip their work (NVLink pull, gradient clear, AdamW
update) and that the trainer raises one step later.
"""
import time

import pytest
import torch

from centrifuge_b200.utils.device_status import DeviceError, DeviceStatus, describe

K_ERR_PEER_WAIT = 32


def test_status_reader_cpu_block():
    block = torch.zeros(4, dtype=torch.int32)
    st = DeviceStatus("cpu", block=block)
    st.record()  # clean step
    block[0] = K_ERR_PEER_WAIT
    with pytest.raises(DeviceError) as ei:
        st.record()
    assert ei.value.code == K_ERR_PEER_WAIT and ei.value.step == 1
    assert int(block[0]) == 0  # reset so the caller can continue
    st.record()
    assert "peer" in describe(K_ERR_PEER_WAIT)


@pytest.fixture
def short_peer_wait():
    from centrifuge_b200.ops._ext import kernels
    k = kernels()
    status = k.status_block(0)
    status.zero_()
    k.set_wait_limits(0, 0, 5000)  # peer waits give up after 5 ms
    try:
        yield k, status
    finally:
        k.set_wait_limits(0, 0, 0)
        status.zero_()
        torch.cuda.synchronize()


@pytest.mark.gpu
def test_peer_wait_times_out_and_later_kernels_skip(short_peer_wait):
    k, status = short_peer_wait
    dev = torch.device("cuda", 0)
    flags = torch.zeros(8, dtype=torch.int32, device=dev)  # nothing ever raises these
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    k.symm_wait(flags.data_ptr(), 0, 1, 1, 1, status)
    torch.cuda.synchronize()
    dt = time.perf_counter() - t0
    assert int(status[0]) == K_ERR_PEER_WAIT
    assert dt < 2.0, f"the wait returned after {dt:.3f} s (limit 5 ms)"

    # the pull after a failed wait leaves the destination untouched
    src = torch.full((1024,), 3.0, device=dev)
    ptrs = torch.tensor([src.data_ptr()], dtype=torch.int64, device=dev)
    dst = torch.ones(1024, device=dev)
    k.symm_pull_reduce(0, ptrs.data_ptr(), 1, 0, 1024, dst, 1.0, status)
    buf = torch.ones(1000, device=dev)
    k.zero_unless_error(buf, status)
    # the clip coefficient marks the step as failed and AdamW leaves everything untouched
    g = torch.ones(4096, device=dev)
    partial = torch.empty(148 * 4, device=dev)
    coef, norm = torch.empty(1, device=dev), torch.empty(1, device=dev)
    k.sumsq(g, partial)
    k.clip_coef(partial, 1.0, 1.0, coef, norm)
    master = torch.randn(4096, device=dev)
    m, v = torch.zeros_like(master), torch.zeros_like(master)
    p = master.to(torch.bfloat16)
    before = (master.clone(), p.clone())
    k.adamw(master, g, m, v, p, 1e-3, 0.9, 0.95, 1e-8, 0.0, 0.1, 0.05, coef)
    torch.cuda.synchronize()
    assert torch.equal(dst, torch.ones_like(dst))
    assert torch.equal(buf, torch.ones_like(buf))
    assert float(coef) == -1.0
    assert torch.equal(master, before[0]) and torch.equal(p, before[1])
    assert float(m.abs().sum()) == 0.0

    # with the word cleared the same kernels do their work
    status[:1].zero_()
    k.symm_pull_reduce(0, ptrs.data_ptr(), 1, 0, 1024, dst, 1.0, status)
    k.zero_unless_error(buf, status)
    k.clip_coef(partial, 1.0, 1.0, coef, norm)
    k.adamw(master, g, m, v, p, 1e-3, 0.9, 0.95, 1e-8, 0.0, 0.1, 0.05, coef)
    torch.cuda.synchronize()
    assert torch.equal(dst, torch.full_like(dst, 4.0))
    assert float(buf.abs().sum()) == 0.0
    assert 0.0 < float(coef) <= 1.0
    assert not torch.equal(master, before[0])


@pytest.mark.gpu
def test_trainer_raises_one_step_after_a_failed_wait(short_peer_wait, tmp_path, monkeypatch):
    from centrifuge_b200.config import tiny_llama_test
    from centrifuge_b200.data.synthetic import SyntheticTokenData
    from centrifuge_b200.models.llama import NativeLlamaForCausalLM
    from centrifuge_b200.parallel.zero import ZeroAdamW
    from centrifuge_b200.trainer import Trainer

    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    k, status = short_peer_wait
    dev = torch.device("cuda", 0)
    cfg = tiny_llama_test(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=1024,
                          head_dim=64)
    model = NativeLlamaForCausalLM(cfg, device=dev, seed=0)
    opt = ZeroAdamW(model.flat, group=None, stage=2, lr=1e-3, betas=(0.9, 0.95), eps=1e-8,
                    weight_decay=0.0, grad_clip=1.0, reducer=None)
    tr = Trainer(model, opt, drop_rate=0.5, grad_accum=1, world_size=1)
    data = SyntheticTokenData(cfg.vocab_size, 2, 128, seed=1, rank=0)
    batch = [data.sample().to(dev)]
    tr.train_step(batch, to_device=False)  # clean step 0

    flags = torch.zeros(8, dtype=torch.int32, device=dev)
    k.symm_wait(flags.data_ptr(), 0, 1, 1, 1, status)  # runs out between steps
    before = model.flat.data.clone()
    tr.train_step(batch, to_device=False)  # step 1: update skipped on the device
    torch.cuda.synchronize()
    assert torch.equal(model.flat.data, before), "the failed step must not update parameters"
    with pytest.raises(DeviceError) as ei:
        tr.train_step(batch, to_device=False)  # step 2 reads step 1's word
    assert ei.value.code == K_ERR_PEER_WAIT and ei.value.step == 1
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    tr.train_step(batch, to_device=False)  # training can continue after handling it
    tr.status.check_now()
    assert not torch.equal(model.flat.data, before)


@pytest.mark.gpu
def test_out_of_range_indices_are_recorded_not_read():
    """A token id past the vocabulary, a row id past the table and a label past the vocabulary
    are recorded in the status word (kErrBounds) and skipped: zero rows / zero loss, no fault."""
    from centrifuge_b200.ops import fused
    from centrifuge_b200.ops._ext import kernels
    k = kernels()
    status = k.status_block(0)
    status.zero_()
    dev = torch.device("cuda", 0)
    V, H = 64, 128
    table = torch.randn(V, H, device=dev).bfloat16()
    ids = torch.tensor([3, V, 5, V + 1000], device=dev)
    out = fused.embedding_fwd(table, ids)
    torch.cuda.synchronize()
    assert int(status[0]) == 128
    assert torch.equal(out[0], table[3]) and torch.equal(out[2], table[5])
    assert float(out[1].float().abs().sum()) == 0.0 and float(out[3].float().abs().sum()) == 0.0
    status.zero_()
    rows = torch.tensor([1, -1, V], dtype=torch.int32, device=dev)
    g = fused.gather_rows(table, rows)
    torch.cuda.synchronize()
    assert int(status[0]) == 128
    assert torch.equal(g[0], table[1]) and float(g[1:].float().abs().sum()) == 0.0
    status.zero_()
    logits = torch.randn(4, V, device=dev).bfloat16()
    labels = torch.tensor([1, V, -100, 2], device=dev)
    loss, _ = fused.ce_fwd(logits, labels)
    torch.cuda.synchronize()
    assert int(status[0]) == 128
    assert float(loss[1]) == 0.0 and float(loss[2]) == 0.0 and float(loss[0]) > 0.0
    status.zero_()
    # embedding gradient: token V (out of range) and row id 9 (past ids) are skipped
    dy = torch.randn(3, H, device=dev).bfloat16()
    for det in (True, False):
        dt = torch.zeros(V, H, device=dev)
        fused.embedding_bwd(dy, ids, dt, torch.tensor([0, 1, 9], dtype=torch.int32, device=dev),
                            deterministic=det)
        torch.cuda.synchronize()
        assert int(status[0]) == 128
        assert torch.equal(dt[3], dy[0].float()) and float(dt.abs().sum()) == float(
            dy[0].float().abs().sum())
        status.zero_()
    torch.cuda.synchronize()
