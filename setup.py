"""Builds the sm_100a kernel library in-tree: `python setup.py build_ext --inplace`.

All CUDA sources under miles_b200/csrc are compiled for sm_100a only (tcgen05 / TMA kernels do
not exist on other architectures) and linked into one extension, miles_b200._C.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("miles_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("MILES_B200_CHECKS") == "1":
    NVCC_FLAGS.append("-DMB_CHECKS=1")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))

setup(
    name="miles_b200",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="miles_b200._C",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
