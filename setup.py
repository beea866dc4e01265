"""Builds the abacus_b200._C extension (hand-written sm_100a kernels) in-tree.

    python setup.py build_ext --inplace

Every CUDA source is compiled for sm_100a only (tcgen05 / TMA / TMEM).
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))

# Link libstdc++ dynamically: a toolchain that silently falls back to the
# static archive puts a second libstdc++ into the process next to torch's, and
# stream formatting (e.g. error messages) then crashes on non-main threads.
for var, exe in (("CXX", "/usr/bin/g++"), ("CC", "/usr/bin/gcc")):
    if os.path.exists(exe):
        os.environ[var] = exe
CSRC = os.path.join("abacus_b200", "csrc")

sources = sorted(
    glob.glob(os.path.join(CSRC, "**", "*.cu"), recursive=True)
    + glob.glob(os.path.join(CSRC, "**", "*.cpp"), recursive=True)
)

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("ABACUS_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "-DNDEBUG",
]

setup(
    name="abacus_b200",
    version="0.1.0",
    packages=["abacus_b200"],
    ext_modules=[
        CUDAExtension(
            name="abacus_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
