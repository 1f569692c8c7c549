"""Builds the package's sm_100a CUDA extension in place:

    python setup.py build_ext --inplace

Every kernel is compiled for Blackwell data-center parts only
(-gencode arch=compute_100a,code=sm_100a); nothing else is targeted.
"""
import glob
import os

from setuptools import setup

os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
from torch.utils.cpp_extension import BuildExtension, CUDAExtension  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("vdn_minimax_h3_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("VDN_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]


def extension():
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "ops.cpp")]
    return CUDAExtension(
        name="vdn_minimax_h3_b200._C",
        sources=sources,
        include_dirs=[os.path.join(HERE, CSRC)],
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    )


setup(
    name="vdn_minimax_h3_b200",
    version="0.1.0",
    packages=["vdn_minimax_h3_b200"],
    ext_modules=[extension()],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
