"""Builds the sm_100a extension in-tree: `python setup.py build_ext --inplace`.

Every kernel is compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`); torch's
own arch list is bypassed.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("dllm_qwen38_b200", "csrc")
SOURCES = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
NVCC = [
    "-O3", "-lineinfo", "-std=c++17",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "--expt-relaxed-constexpr", "-Xptxas=-v" if os.environ.get("BDLLM_PTXAS_V") else "-Xptxas=-O3",
    "-DNDEBUG",
]

setup(
    name="dllm_qwen38_b200",
    version="0.1.0",
    packages=["dllm_qwen38_b200"],
    ext_modules=[
        CUDAExtension(
            "dllm_qwen38_b200._C",
            SOURCES,
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
        )
    ],
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
