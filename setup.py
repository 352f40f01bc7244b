"""Build the sm_100a kernel library in-tree:  python setup.py build_ext --inplace

Every CUDA translation unit is compiled for sm_100a only (tcgen05 / TMEM / TMA need the
arch-specific target); the torch bindings live in one C++ file.
"""
import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("tensor_train_ing_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("TTB_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__", "-U__CUDA_NO_HALF2_OPERATORS__",
]


def sources():
    cu = sorted(glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True))
    return [os.path.join(CSRC, "bindings.cpp")] + cu


setup(
    name="tensor_train_ing_b200",
    version="0.1.0",
    packages=find_packages(include=["tensor_train_ing_b200*"]),
    ext_modules=[
        CUDAExtension(
            name="tensor_train_ing_b200._C",
            sources=sources(),
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
    entry_points={"console_scripts": ["tnlm = tensor_train_ing_b200.cli:main"]},
)
