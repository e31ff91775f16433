"""In-tree build of the sm_100a extensions.

    python setup.py build_ext --inplace

builds ``primus_dlrm_b200/_C*.so`` (core kernels) and
``primus_dlrm_b200/_gemm*.so`` (tcgen05 GEMM / attention kernels) next to
the package, so the shared objects travel with the source tree.  Every CUDA
source is compiled for ``sm_100a`` only.
"""
from __future__ import annotations

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


NVCC_COMMON = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "--expt-extended-lambda",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT162_OPERATORS__", "-U__CUDA_NO_BFLOAT162_CONVERSIONS__",
]
CXX = ["-O3", "-std=c++17"]

core_sources = ["csrc/bindings.cpp"] + sorted(
    s for s in glob.glob("csrc/*.cu") if not os.path.basename(s).startswith("gemm")
    and not os.path.basename(s).startswith("attn"))
gemm_sources = sorted(glob.glob("csrc/gemm*.cu") + glob.glob("csrc/attn*.cu")) + ["csrc/gemm_bindings.cpp"]

ext_modules = [
    CUDAExtension(
        name="primus_dlrm_b200._C",
        sources=core_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={"cxx": CXX, "nvcc": NVCC_COMMON},
    ),
]
if os.path.exists(os.path.join(ROOT, "csrc", "gemm_bindings.cpp")):
    ext_modules.append(CUDAExtension(
        name="primus_dlrm_b200._gemm",
        sources=gemm_sources,
        include_dirs=[os.path.join(ROOT, "csrc")],
        extra_compile_args={
            "cxx": CXX,
            "nvcc": NVCC_COMMON + ["--use_fast_math",
                                   "-Xptxas=-v" if os.environ.get("PD_PTXAS_V") else "-DPD_NOV"],
        },
    ))

setup(
    name="primus_dlrm_b200",
    version="0.1.0",
    packages=["primus_dlrm_b200"],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
