"""Fake (meta) kernels of the token_filter operators (reference grad_filter/token_filter/
ops.py:45-55): tracers such as torch.compile's FakeTensorMode see shape-only results, while real
tensors still reach the graph rewriter."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from centrifuge_b200 import filter as F


def test_fake_tensor_mode_uses_fake_kernels():
    F.load()
    with FakeTensorMode():
        x = torch.randn(4, 8, requires_grad=True)
        loss = (x * 2).sum()
        mask = torch.ones(2, 8, dtype=torch.long)
        out = torch.ops.token_filter.backward_filter.default(loss, mask)
        assert out.shape == loss.shape and out.dtype == loss.dtype
        assert torch.ops.token_filter.backward_filter_with_dims.default(loss, mask, "") == ""
        assert list(torch.ops.token_filter.collect_node_names.default(loss)) == []


def test_meta_tensors_use_fake_kernels():
    F.load()
    loss = torch.empty((), device="meta", requires_grad=True)
    mask = torch.ones(2, 8, dtype=torch.long, device="meta")
    out = torch.ops.token_filter.backward_filter.default(loss, mask)
    assert out.is_meta and out.shape == ()


def test_real_tensors_still_reach_the_rewriter():
    x = torch.randn(4, requires_grad=True)
    loss = (x * 2).sum()
    names = F.collect_node_names(loss)
    assert "MulBackward0" in names and "SumBackward0" in names
