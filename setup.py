"""Builds the sm_100a extensions in-tree: `python setup.py build_ext --inplace`.

`_C` is the library; `_C_dbg` is the same sources compiled with -DBDLLM_DEBUG_BOUNDS (device-side
index / alignment / non-finite checks that record instead of trapping; skip it with
BDLLM_DEBUG_EXT=0). Every kernel is compiled for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`); torch's own arch list is bypassed.
"""

import glob
import os

from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("dllm_qwen38_b200", "csrc")
SOURCES = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
DBG = os.path.join(CSRC, "debug_bounds")


def debug_sources():
    """One wrapper per source under csrc/debug_bounds/ that defines BDLLM_DEBUG_BOUNDS and includes
    it, so the `_C_dbg` objects get their own paths in the build tree (rewritten only on change)."""
    os.makedirs(DBG, exist_ok=True)
    out = []
    for src in SOURCES:
        name = os.path.basename(src)
        text = (f"// Debug-bounds build of ../{name}: the same source compiled with BDLLM_DEBUG_BOUNDS\n"
                f"// (index, alignment and non-finite checks; records read by bounds_report()).\n"
                f"#define BDLLM_DEBUG_BOUNDS 1\n#include \"../{name}\"\n")
        path = os.path.join(DBG, name)
        if not os.path.exists(path) or open(path).read() != text:
            with open(path, "w") as f:
                f.write(text)
        out.append(path)
    return out

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
    ] + ([] if os.environ.get("BDLLM_DEBUG_EXT", "1") == "0" else [
        CUDAExtension(  # the debug-bounds build, loaded under BDLLM_DEBUG_BOUNDS=1
            "dllm_qwen38_b200._C_dbg",
            debug_sources(),
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC},
        )
    ]),
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
