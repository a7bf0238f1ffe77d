"""Build the in-tree sm_100a extension: ``python setup.py build_ext --inplace``."""

import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("uno_b200", "ops", "csrc")
SOURCES = [
    os.path.join(CSRC, name)
    for name in ("bindings.cpp", "gemm_tcgen05.cu", "gemm_noalloc.cu", "attention.cu", "attention_tc.cu", "elementwise.cu",
                 "sampling.cu", "filtered.cu", "comm.cu", "vocab_parallel.cu", "optim.cu", "train_loss.cu", "train_attention.cu", "train_elementwise.cu")
]

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v" if os.environ.get("UNO_PTXAS_VERBOSE") else "-O3",
]

setup(
    name="uno_b200",
    version="0.1.0",
    packages=["uno_b200"],
    ext_modules=[
        CUDAExtension(
            name="uno_b200._C",
            sources=SOURCES,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
            libraries=["cuda"],
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
