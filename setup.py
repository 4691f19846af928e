"""Builds the sm_100a extension in place: ``python setup.py build_ext --inplace``
produces ``afd_demo_b200/_C*.so`` next to the Python package (the extension
is never installed into site-packages).

Only ``-gencode arch=compute_100a,code=sm_100a`` is emitted: the kernels use
tcgen05 / TMA instructions that exist on B200 only, and passing an explicit
-gencode keeps torch from adding its own architecture list.
"""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]
if os.environ.get("AFD_BOUNDS_CHECK"):
    NVCC_FLAGS.append("-DAFD_BOUNDS_CHECK=1")

SOURCES = ["bindings.cpp", "gemm_tcgen05.cu", "gemm_tm.cu", "kernels.cu", "attention.cu",
           "attention_tc.cu", "decode_attention_tc.cu", "noalloc.cu"]

setup(
    name="afd_demo_b200",
    ext_modules=[
        CUDAExtension(
            name="afd_demo_b200._C",
            sources=[os.path.join("csrc", s) for s in SOURCES],
            include_dirs=[CSRC],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
