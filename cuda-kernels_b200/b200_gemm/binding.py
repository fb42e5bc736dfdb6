"""Loader for the prebuilt torch-extension binding (bf16_matmul/matmul.cpp).

The extension is built in-tree by build.py and imported from its file, so no
JIT cache is involved at run time.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util

import torch  # noqa: F401  (the extension links against libtorch)

from .build import EXT_NAME, ext_path

_mod = None


def load_binding():
    """Return the extension module exposing matmul_b200(A, B) and matmul_b200_kn(A, B)."""
    global _mod
    if _mod is None:
        path = ext_path()
        if path is None:
            raise ImportError("torch binding not built; run cuda-kernels_b200/b200_gemm/build.py")
        loader = importlib.machinery.ExtensionFileLoader(EXT_NAME, path)
        spec = importlib.util.spec_from_file_location(EXT_NAME, path, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mod = mod
    return _mod
