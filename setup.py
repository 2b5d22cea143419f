"""Build the native extensions of centrifuge_b200 in-tree.

    python setup.py build_ext --inplace

* ``centrifuge_b200._kernels`` -- the sm_100a CUDA kernels (``-gencode arch=compute_100a,
  code=sm_100a``) and their torch bindings.
* ``centrifuge_b200._filter_C`` -- the C++ autograd-graph rewriter that implements the
  ``token_filter::backward_filter`` / ``backward_filter_with_dims`` / ``collect_node_names``
  operators (built against the installed torch's autograd headers).

The CUDA architecture is fixed to sm_100a: nvcc cross-compiles without a GPU, so this builds on a
CPU-only machine too.
"""
import glob
import os

from setuptools import setup

os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"

from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "centrifuge_b200")
CSRC = os.path.join(PKG, "csrc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("CFB_PTXAS_VERBOSE") == "1" else "-Xptxas=-O3",
    "-DNDEBUG",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-DNDEBUG"]


def kernel_sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    srcs.append(os.path.join(CSRC, "bindings.cpp"))
    return [os.path.relpath(s, ROOT) for s in srcs]


def rewriter_sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "rewriter", "*.cpp")))
    return [os.path.relpath(s, ROOT) for s in srcs]


ext_modules = [
    CUDAExtension(
        "centrifuge_b200._kernels",
        kernel_sources(),
        include_dirs=[CSRC],
        extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
    ),
]
if rewriter_sources():
    ext_modules.append(
        CppExtension(
            "centrifuge_b200._filter_C",
            rewriter_sources(),
            include_dirs=[os.path.join(CSRC, "rewriter")],
            extra_compile_args={"cxx": CXX_FLAGS},
        ))

setup(
    name="centrifuge_b200",
    version="0.1.0",
    packages=["centrifuge_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
