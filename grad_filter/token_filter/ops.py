"""``token_filter.ops``: the reference's one-line entry point, same signatures.

    from grad_filter import token_filter
    token_filter.ops.backward_filter(loss, ref_mask)
"""
from centrifuge_b200.filter import (backward_filter, backward_filter_with_dims,  # noqa: F401
                                    collect_node_names)

__all__ = ["backward_filter", "backward_filter_with_dims", "collect_node_names"]
