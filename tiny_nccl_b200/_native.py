"""Loader for the native extension (``_C``) and its shared libraries.

The extension is built in-tree by ``tiny_nccl_b200/_build.py`` (``build()`` in
``__graft_entry__.py`` runs it). If it is missing at import time and a CUDA
toolchain is present, it is built on the spot; otherwise the import fails with
an explicit error. There is no pure-Python fallback for any collective or
kernel: a missing extension is an error, never a silent CPU path.
"""
from __future__ import annotations

import importlib
import os
import shutil

_C = None


def load():
    global _C
    if _C is not None:
        return _C
    import torch  # noqa: F401  (loads libc10/libtorch before the extension)

    try:
        _C = importlib.import_module("tiny_nccl_b200._C")
    except ImportError as first:
        if os.environ.get("TNCCL_NO_BUILD") or shutil.which("nvcc") is None and not os.path.exists(
                "/usr/local/cuda/bin/nvcc"):
            raise ImportError(f"tiny_nccl_b200 native extension is not built: {first}") from first
        from tiny_nccl_b200 import _build

        _build.build_all()
        _C = importlib.import_module("tiny_nccl_b200._C")
    return _C


def library_path(name: str = "libtnccl.so") -> str:
    """Absolute path of one of the in-tree shared libraries."""
    return os.path.join(os.path.dirname(__file__), "lib", name)
