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
sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))


def _ext(name, extra_defines=()):
    defs = [f"-D{d}" for d in extra_defines]
    return CUDAExtension(
        name=name,
        sources=sources,
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"] + defs, "nvcc": NVCC_FLAGS + defs},
    )


def _checked_sources():
    """One-line wrappers (#define MB_CHECKS + #include of the real source) under build/, so the
    checked objects get their own paths next to the regular ones."""
    out_dir = os.path.join(HERE, "build", "checked_src")
    os.makedirs(out_dir, exist_ok=True)
    out = []
    for src in sources:
        dst = os.path.join(out_dir, os.path.basename(src))
        text = f'#define MB_CHECKS 1\n#include "{os.path.join(HERE, src)}"\n'
        if not os.path.exists(dst) or open(dst).read() != text:
            with open(dst, "w") as f:
                f.write(text)
        out.append(os.path.relpath(dst, HERE))
    return out


# miles_b200._C: the library. miles_b200._C_checked: the same sources with MB_CHECKS=1 (bounds
# guards that record an error code and skip the access; used by the checked-build GPU test).
ext_modules = [_ext("miles_b200._C")]
if os.environ.get("MILES_B200_SKIP_CHECKED") != "1":
    ck = _ext("miles_b200._C_checked")
    ck.sources = _checked_sources()
    ext_modules.append(ck)

setup(
    name="miles_b200",
    packages=[],
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
