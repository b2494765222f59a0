"""In-tree build of the gpt2_harness_b200 native library.

    python setup.py build_ext --inplace

compiles every CUDA source under csrc/ for sm_100a only (B200) and drops
gpt2_harness_b200/_C*.so next to the Python package, where the package imports
it from. Nothing is installed into site-packages.
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")

SOURCES = [
    "csrc/bindings.cpp",
    "csrc/gemm.cu",
    "csrc/attention.cu",
    "csrc/attention_tc.cu",
    "csrc/attention_bwd_tc.cu",
    "csrc/elementwise.cu",
    "csrc/comm.cu",
    "csrc/noalloc.cu",
    "csrc/decode.cu",
    "csrc/zero.cu",
    "csrc/tp.cu",
]

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__",
]

setup(
    name="gpt2_harness_b200",
    version="0.1.0",
    packages=[],
    ext_modules=[
        CUDAExtension(
            name="gpt2_harness_b200._C",
            sources=SOURCES,
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
