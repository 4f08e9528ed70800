"""Build of the sm_100a CUDA extension ``economize_b200._C`` (in-tree: ``python setup.py build_ext --inplace``)."""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "economize_b200", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("ECZ_PTXAS_VERBOSE") else "-O3",
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
sources = [os.path.relpath(s, HERE) for s in sources]

setup(
    name="economize_b200",
    version="0.1.0",
    packages=find_packages(include=["economize_b200", "economize_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="economize_b200._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
