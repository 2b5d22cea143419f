"""Loader of the compiled sm_100a kernel module ``centrifuge_b200._kernels``.

The module is built in-tree by ``python setup.py build_ext --inplace``.  When a CUDA device is
present and the module is missing, every kernel call raises: the GPU path never falls back to a
PyTorch implementation.
"""
from __future__ import annotations

import importlib

_mod = None
_err = None


def kernels():
    """Return the compiled kernel module or raise ``RuntimeError`` naming the build command."""
    global _mod, _err
    if _mod is None and _err is None:
        try:
            _mod = importlib.import_module("centrifuge_b200._kernels")
        except ImportError as e:  # pragma: no cover - depends on the build
            _err = e
    if _mod is None:
        raise RuntimeError(
            "centrifuge_b200._kernels is not built; run `python setup.py build_ext --inplace` "
            f"({_err})")
    return _mod


def available() -> bool:
    try:
        kernels()
        return True
    except RuntimeError:
        return False
