"""Builds the in-tree sm_100a extension ``saint_llm_b200._C``.

    python setup.py build_ext --inplace

Every CUDA source is compiled for ``sm_100a`` only (``-gencode
arch=compute_100a,code=sm_100a``); torch's own arch list is bypassed.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + sorted(glob.glob(os.path.join("csrc", "*.cpp")))

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("SV4_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
os.environ.setdefault("MAX_JOBS", str(max(4, (os.cpu_count() or 8))))

setup(
    name="saint_llm_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="saint_llm_b200._C",
            sources=SOURCES,
            include_dirs=[os.path.join(HERE, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
