"""Loader of the compiled sm_100a kernel module ``centrifuge_b200._kernels``.

The module is built in-tree by ``python setup.py build_ext --inplace``.  When a CUDA device is
present and the module is missing, every kernel call raises: the GPU path never falls back to a
PyTorch implementation.
"""
from __future__ import annotations

import importlib

_mod = None
_err = None
_proxy = None

# Kernels launched by one call of each binding (for the launch counter).
_LAUNCHES_PER_CALL = {"rmsnorm_bwd": 2, "attn_bwd": 2, "attn_bwd_mma": 3, "gemm_error_word": 0,
                      "status_block": 0, "set_wait_limits": 0, "gemm_plan": 0}


class LaunchCounter:
    """Counts sm_100a kernel launches issued through the bindings."""

    def __init__(self):
        self.count = 0

    def reset(self) -> int:
        n, self.count = self.count, 0
        return n


counter = LaunchCounter()


class _Counted:
    def __init__(self, mod):
        self._mod = mod

    def __getattr__(self, name):
        fn = getattr(self._mod, name)
        if not callable(fn):
            return fn
        n = _LAUNCHES_PER_CALL.get(name, 1)

        def call(*args, **kwargs):
            counter.count += n
            return fn(*args, **kwargs)

        setattr(self, name, call)
        return call


def kernels():
    """Return the compiled kernel module or raise ``RuntimeError`` naming the build command."""
    global _mod, _err, _proxy
    if _mod is None and _err is None:
        try:
            _mod = importlib.import_module("centrifuge_b200._kernels")
            _proxy = _Counted(_mod)
        except ImportError as e:  # pragma: no cover - depends on the build
            _err = e
    if _mod is None:
        raise RuntimeError(
            "centrifuge_b200._kernels is not built; run `python setup.py build_ext --inplace` "
            f"({_err})")
    return _proxy


def available() -> bool:
    try:
        kernels()
        return True
    except RuntimeError:
        return False


def status_block(device=None):
    """The kernels' per-device status block (error word + wait limits) of ``device`` (a
    ``torch.device``, an index, or None for the current CUDA device)."""
    import torch
    if device is None:
        idx = torch.cuda.current_device()
    elif isinstance(device, int):
        idx = device
    else:
        d = torch.device(device)
        idx = d.index if d.index is not None else torch.cuda.current_device()
    return kernels().status_block(idx)
