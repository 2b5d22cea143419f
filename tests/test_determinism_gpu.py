"""Run-to-run determinism of the native training step on one B200.

Every kernel of the step reduces in a fixed order (attention accumulators in TMEM, column sums
of the norm weights, the sorted-run embedding gradient, per-block grad-norm partials) except the
split-K weight-gradient GEMMs, whose partial tiles meet in fp32 vector reductions in arrival
order.  With split-K off (CFB_GEMM_SPLIT_K=0, read once per process, hence the child process)
two identical training runs give the same bits.
"""
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = r"""
import sys, torch
sys.path.insert(0, sys.argv[1])
from centrifuge_b200.config import tiny_llama_test
from centrifuge_b200.data.synthetic import Batch
from centrifuge_b200.models.llama import NativeLlamaForCausalLM
from centrifuge_b200.parallel.zero import ZeroAdamW
from centrifuge_b200.trainer import Trainer

def run():
    cfg = tiny_llama_test(layers=2, hidden=256, heads=4, kv_heads=2, ffn=512, vocab=1024,
                          head_dim=64)
    model = NativeLlamaForCausalLM(cfg, device="cuda", seed=0)
    init = model.flat.data.clone()
    opt = ZeroAdamW(model.flat, lr=1e-3, grad_clip=1.0)
    tr = Trainer(model, opt, drop_rate=0.5, grad_accum=2)
    g = torch.Generator().manual_seed(5)
    for _ in range(2):
        bs = [Batch(torch.randint(0, cfg.vocab_size, (2, 256), generator=g),
                    torch.exp(1.0 + 0.5 * torch.randn(2, 255, generator=g))) for _ in range(2)]
        tr.train_step(bs)
    torch.cuda.synchronize()
    return model.flat.data.clone(), opt.master.clone(), init

a, b = run(), run()
same = torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
moved = not torch.equal(a[0], a[2])
print("RESULT", "same" if same else "different", "trained" if moved else "untrained")
"""


def test_training_step_bitwise_deterministic():
    env = dict(os.environ, CFB_GEMM_SPLIT_K="0")
    out = subprocess.run([sys.executable, "-c", CHILD, ROOT], env=env, capture_output=True,
                         text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = [ln for ln in out.stdout.splitlines() if ln.startswith("RESULT")][-1]
    assert line == "RESULT same trained", line
