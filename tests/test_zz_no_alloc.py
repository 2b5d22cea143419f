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


def _call(lib, dy, x, rows, rstd, w, dres, dx, dw, R, H):
    stream = torch.cuda.current_stream().cuda_stream
    return lib.cfb_rmsnorm_bwd_noalloc(_ptr(dy), _ptr(x), _ptr(rows), _ptr(rstd), _ptr(w),
                                       _ptr(dres), _ptr(dx), _ptr(dw), R, H,
                                       ctypes.c_void_p(stream))


# (T rows of x, H, R rows of dy, gathered rows?).  H=2048 R=120: one row per block.
# H=8192 R=1000: the scratch caps the partial rows at 2^20 / 8192 = 128, several rows per block.
# H=4096 R=700: 256 partial rows, blocks of 3 rows and idle trailing blocks that write zero
# partial sums.  H=64 R=1: a single row, one group of 8 columns.
CASES = [(300, 2048, 120, True), (1200, 8192, 1000, True), (700, 4096, 700, False),
         (5, 64, 1, True)]


@pytest.mark.parametrize("T,H,R,gather", CASES)
def test_noalloc_matches_regular_entry_point_twice(T, H, R, gather):
    from centrifuge_b200.ops import fused
    from centrifuge_b200.ops import reference as ref
    lib = _lib()
    torch.manual_seed(H + R)
    x = torch.randn(T, H, device="cuda").bfloat16()
    w = (1 + 0.1 * torch.randn(H, device="cuda")).bfloat16()
    _, rstd = fused.rmsnorm_fwd(x, w, 1e-5)
    rows = torch.randperm(T, device="cuda")[:R].sort().values.int() if gather else None
    dw0 = torch.randn(H, device="cuda")  # the entry point accumulates into dw
    for call in range(2):  # two calls in a row share the scratch array
        dy = torch.randn(R, H, device="cuda").bfloat16()
        dres = torch.randn(R, H, device="cuda").bfloat16() if call == 0 else None
        dw_ref = dw0.clone()
        dx_ref = fused.rmsnorm_bwd(dy, x, rstd, w, dw_ref, x_rows=rows, dres=dres)
        dw = dw0.clone()
        dx = torch.empty_like(dy)
        rc = _call(lib, dy, x, rows, rstd, w, dres, dx, dw, R, H)
        assert rc == 0, lib.cfb_noalloc_strerror(rc)
        torch.cuda.synchronize()
        # against the regular entry point
        assert _rel(dx, dx_ref) < 1e-2
        assert _rel(dw - dw0, dw_ref - dw0) < 1e-3
        # against the fp32 definition
        xs = x if rows is None else x[rows.long()]
        rs = rstd if rows is None else rstd[rows.long()]
        dx32, dw32 = ref.rmsnorm_bwd(dy, xs, rs, w, dres)
        assert _rel(dx, dx32) < 1e-2
        assert _rel(dw - dw0, dw32) < 1e-3


def test_noalloc_rejects_misaligned_buffers():
    lib = _lib()
    H, R = 256, 4
    x = torch.randn(R, H, device="cuda").bfloat16()
    w = torch.ones(H, device="cuda").bfloat16()
    rstd = torch.ones(R, device="cuda")
    dy = torch.randn(R * H + 8, device="cuda").bfloat16()
    dx = torch.empty(R, H, device="cuda").bfloat16()
    dw = torch.zeros(H, device="cuda")
    off = ctypes.c_void_p(dy.data_ptr() + 2)  # 2 bytes past a 16-byte boundary
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.cfb_rmsnorm_bwd_noalloc(off, _ptr(x), None, _ptr(rstd), _ptr(w), None, _ptr(dx),
                                     _ptr(dw), R, H, stream)
    assert rc == -1 and b"aligned" in lib.cfb_noalloc_strerror(rc)
    torch.cuda.synchronize()
    assert float(dw.abs().sum()) == 0.0


def test_noalloc_rejects_oversized_hidden():
    lib = _lib()
    z = ctypes.c_void_p(16)
    rc = lib.cfb_rmsnorm_bwd_noalloc(z, z, None, z, z, None, z, z, 4, 16384, None)
    assert rc == -2 and b"8192" in lib.cfb_noalloc_strerror(rc)
