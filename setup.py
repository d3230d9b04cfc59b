"""Builds the in-tree CUDA extension ``elasticmegatron_b200._C`` for sm_100a (B200).

    python setup.py build_ext --inplace
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
SOURCES = sorted(glob.glob(os.path.join("csrc", "**", "*.cu"), recursive=True)) + \
    sorted(glob.glob(os.path.join("csrc", "**", "*.cpp"), recursive=True))

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("EMB_PTXAS_VERBOSE"):
    NVCC_FLAGS += ["-Xptxas", "-v"]
if os.environ.get("EMB_NVCC_EXTRA"):  # extra nvcc flags for experiments, e.g. "-DFA_POLY_MASK=0x5555"
    NVCC_FLAGS += os.environ["EMB_NVCC_EXTRA"].split()

setup(
    name="elasticmegatron_b200",
    packages=[],
    ext_modules=[CUDAExtension(
        name="elasticmegatron_b200._C",
        sources=SOURCES,
        include_dirs=[os.path.join(ROOT, "csrc", "include")],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        libraries=["cuda"],
    )],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
