"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Every CUDA source is compiled for Blackwell only (``-gencode arch=compute_100a,code=sm_100a``); passing our own
``-gencode`` makes torch skip its default architecture list. Kernel sources (``csrc/*.cu``) carry no torch headers,
so they compile in seconds; ``csrc/bindings.cpp`` holds all of the PyTorch glue.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC = ARCH + ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xptxas=-v",
               "-DNDEBUG"]
if os.environ.get("QW_DEBUG_BOUNDS") == "1":
    NVCC.append("-DQW_DEBUG_BOUNDS=1")

sources = sorted(glob.glob(os.path.join("csrc", "*.cu"))) + [os.path.join("csrc", "bindings.cpp")]

setup(
    name="quantaweave_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="quantaweave_b200._C",
            sources=sources,
            include_dirs=[os.path.join(ROOT, "csrc")],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
