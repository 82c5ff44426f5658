"""Builds the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for sm_100a only (tcgen05 / TMA need the
arch-specific target); torch's own arch list is bypassed by passing the
-gencode flag explicitly.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("b200moe", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]

sources = [os.path.join(CSRC, "binding.cpp")] + sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))

setup(
    name="b200moe",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="b200moe._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC, "include")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
