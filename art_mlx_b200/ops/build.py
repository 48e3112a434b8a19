"""Ahead-of-time build of the native extension for sm_100a.

``python -m art_mlx_b200.ops.build`` compiles every ``csrc/*.cu`` / ``*.cpp``
into ``art_mlx_b200/ops/_C.so`` (in-tree, so it ships with the source tree to
the GPU host).  nvcc cross-compiles without a GPU.  At run time the package
imports that file directly; nothing is compiled lazily.
"""

from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
SO_PATH = os.path.join(HERE, "_C.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--use_fast_math",
    "-Xptxas=-v" if os.environ.get("ART_PTXAS_VERBOSE") else "-Xptxas=-O3",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def build(verbose: bool = False) -> str:
    from torch.utils import cpp_extension

    os.makedirs(BUILD_DIR, exist_ok=True)
    # torch's own arch list must not add other targets: the -gencode flags
    # above are the only architecture selection.
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    extra_ldflags: list[str] = []  # no libcuda link: driver entry points are resolved at run time
    mod = cpp_extension.load(
        name="art_b200_C",
        sources=sources(),
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=NVCC_FLAGS,
        extra_ldflags=extra_ldflags,
        extra_include_paths=[CSRC],
        build_directory=BUILD_DIR,
        verbose=verbose,
        is_python_module=True,
    )
    built = mod.__file__
    shutil.copy2(built, SO_PATH + ".tmp")
    os.replace(SO_PATH + ".tmp", SO_PATH)
    return SO_PATH



if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
