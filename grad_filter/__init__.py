"""Compatibility package: ``from grad_filter import token_filter`` as in the reference."""
from . import token_filter  # noqa: F401
