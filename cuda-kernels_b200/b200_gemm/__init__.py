"""b200_gemm — BF16 GEMM for NVIDIA B200 (sm_100a) behind the reference's
bf16_matmul operator API (typr7/CUDA-Kernels, bf16_matmul/matmul.cpp).

    import b200_gemm
    C = b200_gemm.matmul(A, B_nk)              # reference semantics: A @ B.T
    C = b200_gemm.gemm(A, B_kn, b_layout="kn")  # A @ B with B stored [K,N]

Importing the package loads the compiled C-ABI library and fails if it is
missing: there is no fallback path.
"""
from ._lib import B200GemmError, exported_symbols, load as _load_lib
from .ops import check_status, flash_attn, flash_attn_set_kernel, gemm, gemm_f32, matmul, set_kernel, set_timeout_ns

_load_lib()

__all__ = ["B200GemmError", "check_status", "exported_symbols", "flash_attn", "flash_attn_set_kernel", "gemm", "gemm_f32",
           "matmul", "set_kernel", "set_timeout_ns"]
