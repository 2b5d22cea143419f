"""Backward token filtering: the one-line API.

    loss, mask = token_filter_loss(...)          # centrifuge_b200.loss
    backward_filter(loss, mask)                  # rewrite the backward graph of `loss`
    loss.backward()                              # runs on kept tokens only

``backward_filter`` / ``backward_filter_with_dims`` / ``collect_node_names`` are the
``token_filter`` operators (schemas of the reference, grad_filter/token_filter/ops.py:9-39)
implemented by the C++ graph rewriter ``centrifuge_b200._filter_C``.  Native B200 models
(:mod:`centrifuge_b200.models.llama`) are filtered by attaching the mask to their fused backward
node; generic autograd graphs (HuggingFace models) are rewritten node by node.

Dims text (``backward_filter_with_dims``), one block per visited node::

    NodeName
    index bsz_index mode
    ---

``mode``: 0 = B*S, 1 = B*(S-1), 2 = S, 3 = S-1, 4 = none; ``index`` is a dimension or
``a + 10*b`` for two sequence dimensions.  Record it once on a probe batch whose sizes do not
collide with model dimensions (e.g. S=224) and replay it on real batches.
"""
from __future__ import annotations

import importlib
from typing import List

import torch
from torch import Tensor

__all__ = ["backward_filter", "backward_filter_with_dims", "collect_node_names", "load"]

_C = None


def _register_fakes() -> None:
    """FakeTensor (meta) kernels of the three operators, so that ``torch.compile`` and other
    fake-tensor tracers can trace graphs that call them (reference ops.py:45-55): the rewrite
    itself happens at run time; under tracing the loss passes through unchanged in shape."""

    @torch.library.register_fake("token_filter::backward_filter")
    def _fake_backward_filter(loss: Tensor, mask: Tensor) -> Tensor:
        return torch.empty_like(loss)

    @torch.library.register_fake("token_filter::backward_filter_with_dims")
    def _fake_backward_filter_with_dims(loss: Tensor, mask: Tensor, dims: str) -> str:
        return ""

    @torch.library.register_fake("token_filter::collect_node_names")
    def _fake_collect_node_names(loss: Tensor) -> List[str]:
        return []


def load():
    """Import the rewriter extension (registers ``torch.ops.token_filter`` and their fake
    kernels) and the kernels (registers ``torch.ops.cfb`` used by the filtered attention node
    on CUDA)."""
    global _C
    if _C is None:
        mod = importlib.import_module("centrifuge_b200._filter_C")
        _register_fakes()
        _C = mod
        try:
            importlib.import_module("centrifuge_b200._kernels")
        except ImportError:
            if torch.cuda.is_available():
                raise
    return _C


def backward_filter(loss: Tensor, mask: Tensor) -> Tensor:
    """Rewrite ``loss``'s backward graph to run on the kept tokens of ``mask`` ([B, S], 1=keep).

    Dims are cached in ``$CFB_NODE_TRACING_FILE`` (default ``/tmp/node_tracing.txt``) and
    replayed when the cached node sequence matches this graph.
    """
    load()
    return torch.ops.token_filter.backward_filter.default(loss, mask)


def backward_filter_with_dims(loss: Tensor, mask: Tensor, input_node_filter_dims: str = "") -> str:
    """Rewrite with the given dims text (replay) or record them when empty; returns the dims."""
    load()
    return torch.ops.token_filter.backward_filter_with_dims.default(loss, mask,
                                                                   input_node_filter_dims)


def collect_node_names(loss: Tensor) -> List[str]:
    load()
    return list(torch.ops.token_filter.collect_node_names.default(loss))
