"""Efficiency-benchmark driver (reference efficiency_benchmark.py): suites of bench.py runs.

    python -m centrifuge_b200.benchmarks.efficiency --suite fig5b [--gpus 4] [--out results.jsonl]

Modes: ``regular`` (no filtering), ``loss_only`` (filtered loss, dense backward) and
``centrifuge`` (filtered loss and filtered backward).  Suites:

* ``table2``: TinyLlama-1.1B, context 4096, DP=4 (reference: ZeRO-1 DP=4), 50% filter;
* ``fig5a``:  context 1K/2K/3K/4K, regular vs centrifuge;
* ``fig5b``:  filter ratio 20..60%, centrifuge vs regular;
* ``quick``:  one centrifuge run; ``single``: one run of ``--mode``.
Each run is device-timed by bench.py; results are appended as JSON lines.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

FIG5A_CONTEXT = [1024, 2048, 3072, 4096]
FIG5B_DROP = [0.2, 0.3, 0.4, 0.5, 0.6]


def run(gpus: int, mode: str, seq: int, drop: float, steps: int, warmup: int, mbs: int, ga: int,
        model: str = "tinyllama-1.1b", port: int = 29600) -> dict:
    args = ["bench.py", "--gpus", str(gpus), "--steps", str(steps), "--warmup", str(warmup),
            "--mode", mode, "--seq", str(seq), "--drop", str(drop), "--mbs", str(mbs),
            "--ga", str(ga), "--model", model, "--no-e2e"]
    if gpus > 1:
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={gpus}", "--master-addr", "127.0.0.1",
               f"--master-port={port}"] + args
    else:
        cmd = [sys.executable] + args
    out = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
    for line in out.stdout.splitlines():
        if line.startswith("{"):
            return json.loads(line)
    return {"error": out.stderr[-2000:], "cmd": " ".join(cmd)}


def suite_runs(suite: str, mode: str):
    if suite == "table2":
        return [(m, 4096, 0.5) for m in ("regular", "loss_only", "centrifuge")]
    if suite == "fig5a":
        return [(m, s, 0.5) for s in FIG5A_CONTEXT for m in ("regular", "centrifuge")]
    if suite == "fig5b":
        return [("regular", 2048, 0.0)] + [("centrifuge", 2048, d) for d in FIG5B_DROP]
    if suite == "quick":
        return [("centrifuge", 2048, 0.5)]
    return [(mode, 2048, 0.5)]


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--suite", default="quick", choices=["table2", "fig5a", "fig5b", "quick", "single"])
    ap.add_argument("--mode", default="centrifuge", choices=["regular", "loss_only", "centrifuge"])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=2)
    ap.add_argument("--mbs", type=int, default=8)
    ap.add_argument("--ga", type=int, default=4)
    ap.add_argument("--out", default="efficiency_results.jsonl")
    ap.add_argument("--dry-run", action="store_true")
    a = ap.parse_args(argv)
    runs = suite_runs(a.suite, a.mode)
    results = []
    for mode, seq, drop in runs:
        mbs = max(1, a.mbs * 2048 // seq)
        if a.dry_run:
            res = {"mode": mode, "seq": seq, "drop": drop, "mbs": mbs}
        else:
            res = run(a.gpus, mode, seq, drop, a.steps, a.warmup, mbs, a.ga)
            res.update({"suite": a.suite, "mode": mode})
        results.append(res)
        print(json.dumps(res), flush=True)
        if not a.dry_run:
            with open(a.out, "a") as f:
                f.write(json.dumps(res) + "\n")
    return results


if __name__ == "__main__":
    main()
