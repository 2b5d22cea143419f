"""Hot ops of the filtered training step.

On CUDA tensors every op runs a hand-written sm_100a kernel from ``centrifuge_b200._kernels``
(tcgen05/TMEM/TMA GEMM, attention, fused row ops, optimizer, selection).  On CPU tensors they run
the fp32 definitions of :mod:`centrifuge_b200.ops.reference`, which are also the test oracles.
"""
from . import fused, gemm, reference, select  # noqa: F401
from ._ext import available, kernels  # noqa: F401
