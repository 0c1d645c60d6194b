"""Builds the two in-tree extensions of trainium_frontier_b200.

* ``trainium_frontier_b200._native`` - host C++ runtime (data loader); no CUDA.
* ``trainium_frontier_b200._C``      - the sm_100a kernels (tcgen05/TMA/TMEM), built
  only for ``-gencode arch=compute_100a,code=sm_100a``.

Build in place so the shared objects sit next to the Python package:
    python setup.py build_ext --inplace
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CppExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "trainium_frontier_b200")
CSRC = os.path.join(PKG, "csrc")

GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = GENCODE + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get("TFB200_PTXAS_V") else "-Xptxas=-O3",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def rel(paths):
    return sorted(os.path.relpath(p, ROOT) for p in paths)


ext_modules = [
    CppExtension(
        "trainium_frontier_b200._native",
        rel(glob.glob(os.path.join(CSRC, "native", "*.cpp"))),
        extra_compile_args={"cxx": CXX_FLAGS},
    ),
]
if os.environ.get("TFB200_SKIP_CUDA", "0") != "1":
    ext_modules.append(
        CUDAExtension(
            "trainium_frontier_b200._C",
            rel(glob.glob(os.path.join(CSRC, "kernels", "*.cu")) + glob.glob(os.path.join(CSRC, "kernels", "*.cpp"))),
            include_dirs=[os.path.join(CSRC, "kernels")],
            extra_compile_args={"cxx": CXX_FLAGS, "nvcc": NVCC_FLAGS},
        )
    )

setup(
    name="trainium_frontier_b200",
    version="0.1.0",
    packages=["trainium_frontier_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
