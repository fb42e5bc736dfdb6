"""CPU tests of the C-ABI library: it loads, exports every symbol that
include/b200_gemm.h declares, and rejects bad arguments before touching the
GPU (these calls return from the argument checks; no kernel is launched)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "b200_gemm.h")


def _declared():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"B200_API\s+(?:const\s+)?\w+\*?\s+\*?(b200_\w+)\s*\(", txt)))


def test_header_declares_entry_points():
    names = _declared()
    assert "b200_gemm_bf16" in names and "b200_gemm_status" in names
    assert len(names) >= 5


def test_library_exports_every_declared_symbol():
    from b200_gemm import _lib
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), f"{name} declared in include/b200_gemm.h but not exported"
    assert set(_declared()) <= set(_lib.exported_symbols())


def test_version_and_strerror():
    from b200_gemm import _lib
    lib = _lib.load()
    assert b"sm_100a" in lib.b200_gemm_version()
    assert lib.b200_gemm_strerror(0) == b"ok"
    assert lib.b200_gemm_strerror(6).startswith(b"device-side wait")
    assert lib.b200_gemm_strerror(999) == b"unknown error"


def test_argument_errors_without_gpu():
    from b200_gemm import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    fake = P(0x10000)  # never dereferenced: every call below fails its host-side checks first
    # negative size
    assert lib.b200_gemm_bf16(fake, fake, fake, -1, 8, 8, 8, 8, 8, 0, None) == _lib.B200_ERR_INVALID_ARG
    # bad layout
    assert lib.b200_gemm_bf16(fake, fake, fake, 8, 8, 8, 8, 8, 8, 7, None) == _lib.B200_ERR_INVALID_ARG
    # empty output is a no-op
    assert lib.b200_gemm_bf16(fake, fake, fake, 0, 8, 8, 8, 8, 8, 0, None) == _lib.B200_OK
    assert lib.b200_gemm_bf16(fake, fake, fake, 8, 0, 8, 8, 8, 8, 0, None) == _lib.B200_OK
    # null C
    assert lib.b200_gemm_bf16(fake, fake, None, 8, 8, 8, 8, 8, 8, 0, None) == _lib.B200_ERR_INVALID_ARG
    # ldc < N
    assert lib.b200_gemm_bf16(fake, fake, fake, 8, 16, 8, 8, 8, 8, 0, None) == _lib.B200_ERR_INVALID_ARG
    # misaligned C / pitch not a multiple of 8 elements
    assert lib.b200_gemm_bf16(fake, fake, P(0x10002), 8, 8, 8, 8, 8, 8, 0, None) == _lib.B200_ERR_ALIGNMENT
    assert lib.b200_gemm_bf16(fake, fake, fake, 8, 6, 8, 8, 8, 6, 0, None) == _lib.B200_ERR_ALIGNMENT
    # too large
    assert lib.b200_gemm_bf16(fake, fake, fake, 1 << 31, 8, 8, 8, 8, 8, 0, None) == _lib.B200_ERR_TOO_LARGE


def test_product_path_does_not_touch_oracle():
    """The package must not import or load anything under oracle/."""
    pkg = os.path.join(REPO, "cuda-kernels_b200")
    for root, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                txt = open(os.path.join(root, f), errors="ignore").read()
                assert "oracle" not in re.sub(r"#.*|//.*", "", txt).lower() or f == "build.py", f


def test_torch_binding_rejects_bad_arguments_on_cpu():
    """The reference-shaped torch binding raises (never crashes) on bad input;
    these checks run before any CUDA call, so they need no GPU."""
    import torch
    from b200_gemm.binding import load_binding
    ext = load_binding()
    a = torch.zeros((64, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ext.matmul_b200(a, a)
    with pytest.raises(ValueError, match="bfloat16"):
        ext.matmul_b200(a.float(), a)
    with pytest.raises(ValueError, match="bfloat16"):
        ext.matmul_b200_kn(a.half(), a)


def test_attention_binding_rejects_bad_arguments_on_cpu():
    """The reference-shaped attention binding (flash_attn/flash_attn.cpp:16-30)
    exports both names and raises on bad input before any CUDA call."""
    import torch
    from b200_gemm.binding import load_attn_binding
    ext = load_attn_binding()
    assert hasattr(ext, "fa2_tma_lazy_rescale") and hasattr(ext, "flash_attn_b200")
    q = torch.zeros((1, 128, 2, 128), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ext.fa2_tma_lazy_rescale(q, q, q)
    with pytest.raises(ValueError, match="bfloat16"):
        ext.flash_attn_b200(q.float(), q, q, causal=False)
    with pytest.raises(ValueError, match="4-D"):
        ext.fa2_tma_lazy_rescale(q[0], q[0], q[0])


def test_attention_argument_errors_without_gpu():
    """b200_flash_attn_bf16 checks its arguments before touching the device."""
    from b200_gemm import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    fake = P(0x10000)
    f = lib.b200_flash_attn_bf16
    assert f(fake, fake, fake, fake, 1, 128, 2, 2, 64, 1, None) == _lib.B200_ERR_INVALID_ARG   # head_dim 64
    assert f(fake, fake, fake, fake, 1, 128, 6, 4, 128, 1, None) == _lib.B200_ERR_INVALID_ARG  # 6 % 4 != 0
    assert f(fake, fake, fake, fake, 1, 128, 2, 0, 128, 1, None) == _lib.B200_ERR_INVALID_ARG  # no kv heads
    assert f(fake, fake, fake, fake, -1, 128, 2, 2, 128, 1, None) == _lib.B200_ERR_INVALID_ARG
    assert f(fake, fake, fake, fake, 1 << 17, 128, 2, 2, 128, 1, None) == _lib.B200_ERR_TOO_LARGE
    assert f(fake, None, fake, fake, 1, 128, 2, 2, 128, 1, None) == _lib.B200_ERR_INVALID_ARG
    assert f(fake, fake, P(0x10008), fake, 1, 128, 2, 2, 128, 1, None) == _lib.B200_ERR_ALIGNMENT
    assert f(fake, fake, fake, fake, 0, 128, 2, 2, 128, 1, None) == _lib.B200_OK  # empty: nothing to do
    assert lib.b200_flash_attn_set_kernel(3) == _lib.B200_ERR_INVALID_ARG
    assert lib.b200_flash_attn_set_kernel(-1) == _lib.B200_ERR_INVALID_ARG
    assert lib.b200_flash_attn_set_kernel(_lib.B200_ATTN_KERNEL_AUTO) == _lib.B200_OK


def test_epilogue_argument_errors_without_gpu():
    from b200_gemm import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    fake = P(0x10000)
    bad_dtype = _lib.Epilogue(alpha=1.0, beta=0.0, c_in=None, ldc_in=0, bias=None, d_dtype=7)
    assert lib.b200_gemm_bf16_ex(fake, fake, fake, 8, 8, 8, 8, 8, 8, 0, ctypes.byref(bad_dtype),
                                 None) == _lib.B200_ERR_INVALID_ARG
    odd_bias = _lib.Epilogue(alpha=1.0, beta=0.0, c_in=None, ldc_in=0, bias=0x10002, d_dtype=0)
    assert lib.b200_gemm_bf16_ex(fake, fake, fake, 8, 8, 8, 8, 8, 8, 0, ctypes.byref(odd_bias),
                                 None) == _lib.B200_ERR_ALIGNMENT
    no_c = _lib.Epilogue(alpha=1.0, beta=1.0, c_in=None, ldc_in=8, bias=None, d_dtype=0)
    assert lib.b200_gemm_bf16_ex(fake, fake, fake, 8, 8, 8, 8, 8, 8, 0, ctypes.byref(no_c),
                                 None) == _lib.B200_ERR_INVALID_ARG
    short_ld = _lib.Epilogue(alpha=1.0, beta=1.0, c_in=0x20000, ldc_in=4, bias=None, d_dtype=0)
    assert lib.b200_gemm_bf16_ex(fake, fake, fake, 8, 8, 8, 8, 8, 8, 0, ctypes.byref(short_ld),
                                 None) == _lib.B200_ERR_INVALID_ARG
    f32_alias = _lib.Epilogue(alpha=1.0, beta=1.0, c_in=0x10000, ldc_in=8, bias=None, d_dtype=1)
    assert lib.b200_gemm_bf16_ex(fake, fake, fake, 8, 8, 8, 8, 8, 8, 0, ctypes.byref(f32_alias),
                                 None) == _lib.B200_ERR_INVALID_ARG


def test_f32_argument_errors_without_gpu():
    from b200_gemm import _lib
    lib = _lib.load()
    P = ctypes.c_void_p
    fake = P(0x10000)
    n = ctypes.c_size_t(0)
    assert lib.b200_gemm_f32_workspace_bytes(64, 64, 64, 1, ctypes.byref(n)) == _lib.B200_OK
    # 3 bf16 parts x 2 uses each: A' is M x 6K, B' is 6K x N, bf16
    assert n.value == 64 * 384 * 2 + 384 * 64 * 2
    assert lib.b200_gemm_f32(fake, fake, fake, -1, 8, 8, 8, 8, 8, 1, fake, 1 << 20, None) == _lib.B200_ERR_INVALID_ARG
    assert lib.b200_gemm_f32(fake, fake, fake, 8, 8, 8, 8, 8, 8, 5, fake, 1 << 20, None) == _lib.B200_ERR_INVALID_ARG
    assert lib.b200_gemm_f32(fake, fake, P(0x10004), 8, 8, 8, 8, 8, 8, 1, fake, 1 << 20, None) == _lib.B200_ERR_ALIGNMENT
    assert lib.b200_gemm_f32(fake, fake, fake, 8, 8, 8, 8, 8, 8, 1, fake, 16, None) == _lib.B200_ERR_INVALID_ARG
    assert lib.b200_gemm_f32(fake, fake, fake, 8, 8, 8, 8, 8, 8, 1, P(0x10010), 1 << 20, None) == _lib.B200_ERR_ALIGNMENT


def test_bcast_pieces_match_the_documented_layout():
    """b200_bcast_piece (native, host only) cuts the buffer exactly as
    dist.broadcast_chunks documents: world-1 pieces, 256-byte aligned starts."""
    import ctypes
    from b200_gemm import _lib
    from b200_gemm.dist import broadcast_chunks
    lib = _lib.load()
    for world in (2, 3, 5, 8):
        for nbytes in (16, 1000, 32 << 20, (128 << 20) + 258):
            got = []
            for i in range(world - 1):
                off, n = ctypes.c_size_t(), ctypes.c_size_t()
                assert lib.b200_bcast_piece(world, nbytes, i, ctypes.byref(off), ctypes.byref(n)) == _lib.B200_OK
                got.append((off.value, n.value))
            assert got == broadcast_chunks(nbytes, world)
    off, n = ctypes.c_size_t(), ctypes.c_size_t()
    assert lib.b200_bcast_piece(1, 100, 0, ctypes.byref(off), ctypes.byref(n)) == _lib.B200_ERR_INVALID_ARG
    assert lib.b200_bcast_flag_bytes(8) == 4 * (_lib.B200_BCAST_SLOTS * 8 * 1 + 8 + 1)
