"""Builds the sm_100a CUDA extension of nano_gpic_b200 in the source tree.

    python setup.py build_ext --inplace        (or: python -c "import __graft_entry__ as g; g.build()")

Every kernel is compiled for sm_100a only (tcgen05/TMEM/TMA code has no other target); the -gencode flag in the nvcc
arguments keeps torch from adding its own architecture list.
"""
import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("NG_PTXAS_VERBOSE") == "1" else "-Xptxas=-O3",
    "-DNDEBUG",
]


def sources():
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    return [os.path.relpath(s, HERE) for s in srcs]


setup(
    name="nano_gpic_b200",
    version="0.1.0",
    packages=["nano_gpic_b200"],
    ext_modules=[
        CUDAExtension(
            name="nano_gpic_b200._C",
            sources=sources(),
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
