"""Builds the sm_100a extension in place: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for ``compute_100a``/``sm_100a`` only (tcgen05, TMA and
tensor memory are sm_100a features); the extension lands next to its Python package as
``cs244c_llama_zero_b200/ops/_C*.so``.

``ZB_DEBUG_BOUNDS=1 python setup.py build_ext --inplace --build-temp build/debug_bounds`` builds the
debug-bounds variant ``_C_debug`` (``-DB200_DEBUG_BOUNDS``: hand-indexed global accesses are
range-checked, recorded and skipped when out of range); ``ZB_DEBUG_BOUNDS=1`` at run time loads it.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("cs244c_llama_zero_b200", "ops", "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
    "-DNDEBUG",
]

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
DEBUG_BOUNDS = os.environ.get("ZB_DEBUG_BOUNDS", "0") not in ("", "0")
EXT_NAME = "_C_debug" if DEBUG_BOUNDS else "_C"
if DEBUG_BOUNDS:
    NVCC_FLAGS = NVCC_FLAGS + ["-DB200_DEBUG_BOUNDS"]

setup(
    name="cs244c_llama_zero_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name=f"cs244c_llama_zero_b200.ops.{EXT_NAME}",
            sources=sources,
            include_dirs=[os.path.join(HERE, CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
