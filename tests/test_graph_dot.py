"""gen_node_tracing.py --gen_computational_graph: the backward graph as DOT text."""
import os
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def test_backward_graph_dot(tmp_path):
    from gen_node_tracing import gen_graph_with_model

    from centrifuge_b200.config import get_model_config
    from centrifuge_b200.filter.probe import build_hf_model
    torch.manual_seed(0)
    model = build_hf_model(get_model_config("tiny").to_hf_dict(), "sdpa", "cpu")
    ids = torch.randint(0, model.config.vocab_size, (1, 32))
    loss = model(input_ids=ids, labels=ids).loss
    path = gen_graph_with_model(loss, model, str(tmp_path / "g.dot"))
    text = open(path).read()
    assert text.startswith("digraph backward {") and text.rstrip().endswith("}")
    nodes = [ln for ln in text.splitlines() if "[label=" in ln]
    edges = [ln for ln in text.splitlines() if "->" in ln]
    # every parameter is a named leaf, filtered node types are highlighted, the graph is connected
    n_params = sum(1 for _ in model.parameters())
    assert sum("lightblue" in ln for ln in nodes) == n_params
    assert any("orange" in ln and "NllLossBackward0" in ln for ln in nodes)
    assert len(edges) >= len(nodes) - 1
    assert 'label="lm_head.weight' in text
