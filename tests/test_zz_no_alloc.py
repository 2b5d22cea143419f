"""The allocation-free RMSNorm backward entry point, called through its exported C symbol.

For callers that may not allocate device memory (a host framework that owns every device
allocation, or code that must not trigger cudaFree's device-wide synchronisation), the library
exports ``cfb_rmsnorm_bwd_noalloc``: same result as the regular RMSNorm backward, with its
scratch in a fixed device array.  This file is collected last on purpose.
"""
import ctypes
import glob
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _lib():
    paths = glob.glob(os.path.join(ROOT, "centrifuge_b200", "_kernels*.so"))
    assert paths, "centrifuge_b200._kernels is not built"
    lib = ctypes.CDLL(paths[0])
    f = lib.cfb_rmsnorm_bwd_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 8 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    lib.cfb_noalloc_strerror.restype = ctypes.c_char_p
    lib.cfb_noalloc_strerror.argtypes = [ctypes.c_int]
    return lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / (b.float().norm() + 1e-12)).item()


def test_noalloc_matches_regular_entry_point_twice():
    from centrifuge_b200.ops import fused
    lib = _lib()
    torch.manual_seed(0)
    T, H, R = 300, 2048, 120
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    _, rstd = fused.rmsnorm_fwd(x, w, 1e-5)
    rows = torch.randperm(T, device="cuda")[:R].sort().values.int()
    stream = torch.cuda.current_stream().cuda_stream
    for call in range(2):  # two calls in a row share the scratch array
        dy = torch.randn(R, H, device="cuda").bfloat16()
        dres = torch.randn(R, H, device="cuda").bfloat16() if call == 0 else None
        dw_ref = torch.zeros(H, device="cuda")
        dx_ref = fused.rmsnorm_bwd(dy, x, rstd, w, dw_ref, x_rows=rows, dres=dres)
        dw = torch.zeros(H, device="cuda")
        dx = torch.empty_like(dy)
        rc = lib.cfb_rmsnorm_bwd_noalloc(_ptr(dy), _ptr(x), _ptr(rows), _ptr(rstd), _ptr(w),
                                         _ptr(dres), _ptr(dx), _ptr(dw), R, H,
                                         ctypes.c_void_p(stream))
        assert rc == 0, lib.cfb_noalloc_strerror(rc)
        torch.cuda.synchronize()
        assert _rel(dx, dx_ref) < 1e-2
        assert _rel(dw, dw_ref) < 1e-3


def test_noalloc_rejects_oversized_hidden():
    lib = _lib()
    z = ctypes.c_void_p(16)
    rc = lib.cfb_rmsnorm_bwd_noalloc(z, z, None, z, z, None, z, z, 4, 16384, None)
    assert rc == -2 and b"8192" in lib.cfb_noalloc_strerror(rc)
