"""The training entry point on CPU: native and HF paths, checkpoint save + resume."""
import json
import os

import pytest

from centrifuge_b200.train import main


@pytest.mark.parametrize("impl", ["native", "hf"])
def test_train_and_resume(impl, tmp_path, monkeypatch):
    monkeypatch.setenv("HF_HOME", str(tmp_path))
    monkeypatch.setenv("CFB_NODE_TRACING_FILE", str(tmp_path / "dims.txt"))
    base = ["--task", "train", "--model_path", "tiny", "--synthetic_data", "--context_length", "40",
            "--batch_size", "4", "--micro_batch_size", "2", "--dropping_strategy", "fixed",
            "--drop_rate", "0.5", "--attn_filter", "--model_impl", impl, "--save_steps", "2",
            "--eval_steps", "2", "--output_dir", "run", "--model_cache_dir", str(tmp_path / "run")]
    assert main(base + ["--max_steps", "2"]) == 0
    client = json.load(open(tmp_path / "run" / "training_states" / "client_state.json")) \
        if impl == "native" else None
    if impl == "native":
        assert client["completed_steps"] == 2
        assert os.path.exists(tmp_path / "run" / "model.safetensors")
    # resume continues from step 2
    assert main(base + ["--max_steps", "3"]) == 0
    lines = [json.loads(l) for l in open(tmp_path / "run" / "metrics.jsonl")]
    steps = [l["step"] for l in lines if l["name"] == "train/loss/train"]
    assert steps[-1] == 3
