"""Loader of the in-tree native extension ``art_mlx_b200/ops/_C.so``.

The extension is built ahead of time (``python -m art_mlx_b200.ops.build``).
CUDA tensors are only ever processed by these kernels: if the library is
missing on a GPU host, :func:`lib` raises instead of falling back.
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import sys

_HERE = os.path.dirname(os.path.abspath(__file__))
SO_PATH = os.path.join(_HERE, "_C.so")
_lib = None


def available() -> bool:
    return os.path.exists(SO_PATH)


def lib():
    """The loaded extension module (imports ``_C.so`` once)."""
    global _lib
    if _lib is None:
        if not os.path.exists(SO_PATH):
            raise RuntimeError(
                f"native kernels not built: {SO_PATH} is missing; run "
                "`python -m art_mlx_b200.ops.build` (or __graft_entry__.build())"
            )
        import torch  # noqa: F401  (the extension links against libtorch)

        loader = importlib.machinery.ExtensionFileLoader("art_b200_C", SO_PATH)
        spec = importlib.util.spec_from_file_location("art_b200_C", SO_PATH, loader=loader)
        assert spec is not None
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        sys.modules["art_b200_C"] = mod
        _lib = mod
    return _lib
