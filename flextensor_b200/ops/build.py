"""Build the native extension (sm_100a kernels + runtime) in-tree.

The shared object lands in ``flextensor_b200/ops/_build/ft_b200_C*.so`` and is
imported from there by :mod:`flextensor_b200.ops.native`; nothing is installed
into site-packages. ``-gencode arch=compute_100a,code=sm_100a`` is passed
explicitly, which also stops torch from adding its own architecture list.
"""

from __future__ import annotations

import os
import pathlib

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD_DIR = HERE / "_build"
MODULE_NAME = "ft_b200_C"

SOURCES = [
    "bindings.cpp",
    "runtime.cpp",
    "gemm_sm100.cu",
    "norm.cu",
    "attention_sm100.cu",
    "p2p.cu",
    "tp_sm100.cu",
    "moe_sm100.cu",
    "decode_sm100.cu",
]

CUDA_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
CXX_FLAGS = ["-O3", "-std=c++17"]


def build(verbose: bool = False):
    """Compile (incrementally, via ninja) and return the loaded module."""
    from torch.utils.cpp_extension import load

    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    extra = ["-Xptxas=-v"] if os.environ.get("FT_PTXAS_VERBOSE") else []
    return load(
        name=MODULE_NAME,
        sources=[str(CSRC / s) for s in SOURCES],
        build_directory=str(BUILD_DIR),
        extra_cuda_cflags=CUDA_FLAGS + extra,
        extra_cflags=CXX_FLAGS,
        extra_include_paths=[str(CSRC)],
        with_cuda=True,
        verbose=verbose,
    )


def built_library() -> pathlib.Path | None:
    for p in sorted(BUILD_DIR.glob(f"{MODULE_NAME}*.so")):
        return p
    return None


if __name__ == "__main__":
    m = build(verbose=True)
    print(m.__file__ if hasattr(m, "__file__") else m)
