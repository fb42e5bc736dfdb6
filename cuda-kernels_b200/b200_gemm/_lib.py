"""ctypes binding of the C ABI in include/b200_gemm.h.

This is the thin host layer every Python caller (tests, bench, the
row-sharded driver) goes through.  There is no fallback: if the shared
library is missing the import of b200_gemm fails loudly.
"""
from __future__ import annotations

import ctypes
import os

from .build import LIB_PATH

B200_OK = 0
B200_ERR_INVALID_ARG = 1
B200_ERR_ALIGNMENT = 2
B200_ERR_UNSUPPORTED_DEVICE = 3
B200_ERR_CUDA = 4
B200_ERR_TENSOR_MAP = 5
B200_ERR_DEVICE_TIMEOUT = 6
B200_ERR_TOO_LARGE = 7
B200_ERR_SCRATCH_LIMIT = 8

B200_B_NK = 0
B200_B_KN = 1

B200_IPC_HANDLE_BYTES = 64
B200_BCAST_SLOTS = 3

B200_DTYPE_BF16 = 0
B200_DTYPE_F32 = 1

B200_KERNEL_AUTO = 0
B200_KERNEL_SINGLE = 1
B200_KERNEL_PAIR = 2
B200_KERNEL_SKINNY = 3

B200_ATTN_KERNEL_AUTO = 0
B200_ATTN_KERNEL_SINGLE = 1
B200_ATTN_KERNEL_PAIR = 2

class Epilogue(ctypes.Structure):
    """struct b200_epilogue (include/b200_gemm.h)."""
    _fields_ = [("alpha", ctypes.c_float), ("beta", ctypes.c_float), ("c_in", ctypes.c_void_p),
                ("ldc_in", ctypes.c_int64), ("bias", ctypes.c_void_p), ("d_dtype", ctypes.c_int)]


# Every symbol include/b200_gemm.h declares, with its ctypes signature.
_SIGNATURES = {
    "b200_gemm_bf16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                      ctypes.c_int, ctypes.c_void_p]),
    "b200_gemm_bf16_ws": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "b200_gemm_bf16_ex": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                         ctypes.c_int, ctypes.POINTER(Epilogue), ctypes.c_void_p]),
    "b200_gemm_bf16_allgather": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p),
                                                ctypes.c_int, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                                ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]),
    "b200_ipc_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p), ctypes.c_void_p]),
    "b200_ipc_free": (ctypes.c_int, [ctypes.c_void_p]),
    "b200_ipc_open": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p)]),
    "b200_ipc_close": (ctypes.c_int, [ctypes.c_void_p]),
    "b200_copy_async": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "b200_signal_u32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]),
    "b200_wait_u32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]),
    "b200_bcast_piece": (ctypes.c_int, [ctypes.c_int, ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(ctypes.c_size_t),
                                        ctypes.POINTER(ctypes.c_size_t)]),
    "b200_bcast_flag_bytes": (ctypes.c_size_t, [ctypes.c_int]),
    "b200_bcast_create": (ctypes.c_int, [ctypes.c_int, ctypes.c_int, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p),
                                         ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]),
    "b200_bcast_issue": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]),
    "b200_bcast_wait": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "b200_bcast_release": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]),
    "b200_bcast_destroy": (None, [ctypes.c_void_p]),
    "b200_bcast_issue_range": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_size_t,
                                              ctypes.c_size_t, ctypes.c_void_p]),
    "b200_bcast_gemm": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p,
                                       ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                       ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                       ctypes.c_void_p]),
    "b200_gemm_f32_workspace_bytes": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                                     ctypes.POINTER(ctypes.c_size_t)]),
    "b200_gemm_f32": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                     ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]),
    "b200_flash_attn_bf16": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                            ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]),
    "b200_gemm_bf16_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                              ctypes.c_int, ctypes.c_void_p]),
    "b200_gemm_workspace_bytes": (ctypes.c_int, [ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                                 ctypes.POINTER(ctypes.c_size_t)]),
    "b200_gemm_status": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    "b200_gemm_set_timeout_ns": (ctypes.c_int, [ctypes.c_uint64]),
    "b200_gemm_set_kernel": (ctypes.c_int, [ctypes.c_int]),
    "b200_flash_attn_set_kernel": (ctypes.c_int, [ctypes.c_int]),
    "b200_gemm_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint64, ctypes.c_void_p]),
    "b200_gemm_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "b200_gemm_version": (ctypes.c_char_p, []),
}

_lib = None


class B200GemmError(RuntimeError):
    def __init__(self, code: int, what: str = ""):
        self.code = code
        msg = load().b200_gemm_strerror(code).decode()
        super().__init__(f"b200_gemm error {code}: {msg}" + (f" ({what})" if what else ""))


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is not built; run `python cuda-kernels_b200/b200_gemm/build.py` "
                              "(or __graft_entry__.build()) first")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)
