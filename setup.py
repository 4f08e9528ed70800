"""Build of the sm_100a CUDA extension ``economize_b200._C`` (in-tree: ``python setup.py build_ext --inplace``)."""

import glob
import os

from setuptools import find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))

# Build with the distribution's compiler (host code of the .cu files included; ECZ_HOST_CXX overrides). A GCC
# wrapper that images put into CC/CXX links shared objects in which a C++ exception thrown by the extension (every
# TORCH_CHECK that formats its message) crashes the process instead of raising a Python error.
HOST_CXX = os.environ.get("ECZ_HOST_CXX", "/usr/bin/g++")
if os.path.exists(HOST_CXX):
    os.environ["CXX"] = HOST_CXX
    os.environ["CC"] = HOST_CXX.replace("g++", "gcc") if os.path.exists(HOST_CXX.replace("g++", "gcc")) else HOST_CXX
    os.environ["LDSHARED"] = HOST_CXX + " -shared"
CSRC = os.path.join(HERE, "economize_b200", "csrc")

# ECZ_CHECK=1 builds the bounds-checked variant economize_b200._C_check (kernels check the indices they read from
# device memory and report bad ones in the status word); build it into its own temp folder so the two variants'
# objects do not overwrite each other: ECZ_CHECK=1 python setup.py build_ext --inplace --build-temp build/check
CHECKED = os.environ.get("ECZ_CHECK") == "1"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    *(["-ccbin", HOST_CXX] if os.path.exists(HOST_CXX) else []),
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("ECZ_PTXAS_VERBOSE") else "-O3",
    *(["-DECZ_CHECK"] if CHECKED else []),
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
sources = [os.path.relpath(s, HERE) for s in sources]

setup(
    name="economize_b200",
    version="0.1.0",
    packages=find_packages(include=["economize_b200", "economize_b200.*"]),
    ext_modules=[
        CUDAExtension(
            name="economize_b200._C_check" if CHECKED else "economize_b200._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17", *(["-DECZ_CHECK"] if CHECKED else [])],
                                "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
