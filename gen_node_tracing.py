"""Offline validation of the graph rewrite (onboarding step 3, reference gen_node_tracing.py).

    python gen_node_tracing.py --model_path tiny --batch_size 1 --context_length 224 --filter_graph

Builds the model from its config with random weights, runs forward + the filtered loss,
records the per-node dims with ``backward_filter_with_dims(loss, mask, "")`` into
``tmp/node_tracing.txt`` and runs ``loss.backward()`` through the rewritten graph (shape
errors surface as RuntimeError).  ``--gen_computational_graph`` writes the backward graph of
the loss as Graphviz DOT text (``tmp/computational_graph.dot``; the reference renders the same
graph to SVG with torchviz, gen_node_tracing.py:112-128): one node per autograd node with its
saved tensors' shapes, parameters by name, and the node types the filter rewrites
(``target_node_names.yaml``) highlighted.  Render it with any Graphviz installation.
"""
import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from centrifuge_b200.config import get_model_config  # noqa: E402
from centrifuge_b200.filter import backward_filter_with_dims, collect_node_names  # noqa: E402
from centrifuge_b200.filter.probe import align_seq_len, build_hf_model  # noqa: E402
from centrifuge_b200.loss import token_filter_loss  # noqa: E402


def gen_graph_with_model(loss, model, path="tmp/computational_graph.dot", targets=None):
    """Write the autograd graph below ``loss`` as DOT text and return the path."""
    names = {id(p): n for n, p in model.named_parameters()}
    if targets is None:
        try:
            import yaml
            here = os.path.dirname(os.path.abspath(__file__))
            with open(os.path.join(here, "grad_filter", "target_node_names.yaml")) as f:
                targets = set(yaml.safe_load(f)["target_node_names"])
        except Exception:
            targets = set()
    lines = ["digraph backward {", '  graph [ranksep=0.2, nodesep=0.1, rankdir=TB];',
             '  node [shape=box, fontsize=10, fontname="Times New Roman"];']
    # Python wrappers of autograd nodes are created on access: keep them alive so that id()
    # identifies a node for the whole walk
    seen, visited, stack, alive = {}, set(), [loss.grad_fn], []

    def node_id(fn):
        if id(fn) not in seen:
            alive.append(fn)
            seen[id(fn)] = f"n{len(seen)}"
        return seen[id(fn)]

    while stack:
        fn = stack.pop()
        if fn is None or id(fn) in visited:
            continue
        visited.add(id(fn))
        nid = node_id(fn)
        kind = fn.name()
        if kind == "torch::autograd::AccumulateGrad" or hasattr(fn, "variable"):
            var = getattr(fn, "variable", None)
            label = names.get(id(var), "leaf") + (f"\\n{tuple(var.shape)}" if var is not None else "")
            lines.append(f'  {nid} [label="{label}", style=filled, fillcolor=lightblue];')
        else:
            saved = []
            for attr in dir(fn):
                if attr.startswith("_saved_"):
                    try:
                        v = getattr(fn, attr)
                    except Exception:
                        continue
                    if isinstance(v, torch.Tensor):
                        saved.append(f"{attr[7:]}: {tuple(v.shape)}")
            label = "\\n".join([kind] + saved[:6])  # DOT line breaks
            style = ', style=filled, fillcolor=orange' if kind in targets else ""
            lines.append(f'  {nid} [label="{label}"{style}];')
        for nxt, _ in fn.next_functions:
            if nxt is not None:
                lines.append(f"  {node_id(nxt)} -> {nid};")
                stack.append(nxt)
    lines.append("}")
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    with open(path, "w") as f:
        f.write("\n".join(lines) + "\n")
    return path


def gen_node_tracing_with_model_with_dims(model, batch_size, context_length, vocab_size,
                                          input_dims: str = "", device=None):
    """Record (or replay ``input_dims``) the dims on a random batch and validate the backward."""
    device = device or next(model.parameters()).device
    S = align_seq_len(context_length)
    ids = torch.randint(0, vocab_size, (batch_size, S), device=device)
    ref = torch.randn(batch_size, S - 1, device=device)
    logits = model(input_ids=ids).logits
    loss, mask = token_filter_loss(ids, logits, torch.ones(batch_size, S, dtype=torch.long,
                                                           device=device), ref, "fixed", 0.5,
                                   True, True)
    dims = backward_filter_with_dims(loss, mask, input_dims)
    loss.backward()
    model.zero_grad(set_to_none=True)
    return dims


def gen_node_tracing_with_model(model, batch_size, context_length, vocab_size, out_file,
                                device=None):
    dims = gen_node_tracing_with_model_with_dims(model, batch_size, context_length, vocab_size,
                                                 "", device)
    os.makedirs(os.path.dirname(out_file) or ".", exist_ok=True)
    with open(out_file, "w") as f:
        f.write(dims)
    return dims


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model_path", default="tiny")
    ap.add_argument("--batch_size", type=int, default=1)
    ap.add_argument("--context_length", type=int, default=224)
    ap.add_argument("--filter_graph", action="store_true")
    ap.add_argument("--gen_computational_graph", action="store_true")
    ap.add_argument("--attn_impl", default="sdpa", choices=["eager", "sdpa"])
    ap.add_argument("--use_lora", action="store_true")
    ap.add_argument("--out", default="tmp/node_tracing.txt")
    a = ap.parse_args(argv)
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    try:
        cfg = get_model_config(a.model_path).to_hf_dict()
    except KeyError:
        cfg = a.model_path
    model = build_hf_model(cfg, a.attn_impl, dev)
    if a.use_lora:
        from centrifuge_b200.models.lora import apply_lora
        apply_lora(model)
    if a.gen_computational_graph:
        S = align_seq_len(a.context_length)
        ids = torch.randint(0, model.config.vocab_size, (a.batch_size, S), device=dev)
        loss = model(input_ids=ids, labels=ids).loss
        path = gen_graph_with_model(loss, model, os.path.join(os.path.dirname(a.out) or ".",
                                                              "computational_graph.dot"))
        print(f"backward graph written to {path}")
        model.zero_grad(set_to_none=True)
    if not a.filter_graph:
        S = align_seq_len(a.context_length)
        ids = torch.randint(0, model.config.vocab_size, (a.batch_size, S), device=dev)
        loss = model(input_ids=ids, labels=ids).loss
        print("\n".join(collect_node_names(loss)))
        return 0
    dims = gen_node_tracing_with_model(model, a.batch_size, a.context_length,
                                       model.config.vocab_size, a.out, dev)
    print(f"rewrite validated: {dims.count('---')} nodes, dims written to {a.out}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
