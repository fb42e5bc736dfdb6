"""Loaders for the prebuilt torch-extension bindings (bf16_matmul/matmul.cpp and
flash_attn/flash_attn.cpp).

The extensions are built in-tree by build.py and imported from their files, so
no JIT cache is involved at run time.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util

import torch  # noqa: F401  (the extension links against libtorch)

from .build import EXT_NAME, EXTENSIONS, ext_path

_mods: dict = {}


def _load(name: str, ext_dir: str):
    if name not in _mods:
        path = ext_path(name, ext_dir)
        if path is None:
            raise ImportError(f"torch binding {name} not built; run cuda-kernels_b200/b200_gemm/build.py")
        loader = importlib.machinery.ExtensionFileLoader(name, path)
        spec = importlib.util.spec_from_file_location(name, path, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mods[name] = mod
    return _mods[name]


def load_binding():
    """Return the GEMM extension module: matmul_b200(A, B), matmul_b200_kn(A, B), matmul_b200_f32(A, B)."""
    return _load(EXT_NAME, EXTENSIONS[0][1])


def load_attn_binding():
    """Return the attention extension module: flash_attn_b200(Q, K, V, causal=True) and
    fa2_tma_lazy_rescale(Q, K, V) (causal, the reference operator's name)."""
    name, ext_dir, _ = EXTENSIONS[1]
    return _load(name, ext_dir)
