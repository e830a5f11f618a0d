"""Build the pluggy_b200 sm_100a extension in-tree.

    python setup.py build_ext --inplace

Produces ``pluggy_b200/_C*.so`` next to the Python sources. Only sm_100a is
targeted (``-gencode arch=compute_100a,code=sm_100a``); the flags are given in
``extra_compile_args`` so torch's own arch list is not used.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]
if os.environ.get("PLG_PTXAS_VERBOSE"):
    NVCC_FLAGS.append("-Xptxas=-v")

sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + [os.path.join(CSRC, "bindings.cpp")]
sources = [os.path.relpath(s, ROOT) for s in sources]

setup(
    name="pluggy_b200_ext",
    ext_modules=[
        CUDAExtension(
            name="pluggy_b200._C",
            sources=sources,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            libraries=["cuda"],
            library_dirs=["/usr/local/cuda/lib64/stubs"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
