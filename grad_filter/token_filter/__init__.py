"""``token_filter`` compatibility namespace (reference grad_filter/token_filter/__init__.py)."""
from centrifuge_b200.filter import load as _load

_C = _load()
from . import ops  # noqa: E402,F401
