"""Build the native extensions of mini_nangila_b200 in-tree.

    python setup.py build_ext --inplace

* ``mini_nangila_b200._host``: C++17 host library (pybind11, no CUDA): the
  bit-exact codecs, predictors, topology mask, NZCP I/O and the product-format
  oracle.
* ``mini_nangila_b200._cuda``: sm_100a kernels (torch extension), compiled with
  ``-gencode arch=compute_100a,code=sm_100a`` only.
"""
import glob
import platform
import os

import pybind11
from setuptools import Extension, setup

ROOT = os.path.dirname(os.path.abspath(__file__))
HOST_SRCS = sorted(glob.glob(os.path.join("csrc", "host", "*.cpp")))
CUDA_SRCS = sorted(glob.glob(os.path.join("csrc", "cuda", "*.cu")) + glob.glob(os.path.join("csrc", "cuda", "*.cpp")))

# -fno-trapping-math lets the vectorizer if-convert float compares and
# conversions; it changes no value (the library never reads FP exception flags)
HOST_CFLAGS = ["-O3", "-std=c++17", "-ffp-contract=off", "-fno-fast-math", "-fno-trapping-math", "-Wall",
               "-Wno-sign-compare"]
if platform.machine() in ("x86_64", "AMD64"):
    # SSE4.2 baseline (every x86-64 server CPU since 2009): floor / trunc /
    # min / max become single exact instructions instead of libm calls; no
    # FMA contraction (-ffp-contract=off), so results are unchanged
    HOST_CFLAGS.append("-march=x86-64-v2")
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--fmad=true",
    "-Xptxas", "-v",
    "-DNGL_DEVICE_BUILD",
]
# Bounds-checked debug build: NGL_BOUNDS_CHECK=1 python setup.py build_ext --inplace
if os.environ.get("NGL_BOUNDS_CHECK", "0") == "1":
    NVCC_FLAGS.append("-DNGL_BOUNDS_CHECK")

ext_modules = [
    Extension(
        "mini_nangila_b200._host",
        HOST_SRCS,
        include_dirs=[pybind11.get_include(), os.path.join(ROOT, "csrc")],
        extra_compile_args=HOST_CFLAGS,
        language="c++",
    )
]
cmdclass = {}

if os.environ.get("NGL_SKIP_CUDA", "0") != "1" and CUDA_SRCS:
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    ext_modules.append(
        CUDAExtension(
            "mini_nangila_b200._cuda",
            CUDA_SRCS,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17", "-ffp-contract=off"], "nvcc": NVCC_FLAGS},
            libraries=["cuda"],
        )
    )
    cmdclass["build_ext"] = BuildExtension.with_options(use_ninja=True)

setup(
    name="mini_nangila_b200",
    version="0.1.0",
    packages=[],
    ext_modules=ext_modules,
    cmdclass=cmdclass,
)
