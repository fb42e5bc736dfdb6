"""Torch-facing operator API of the B200 BF16 GEMM.

`matmul(A, B)` keeps the reference operator's meaning exactly: the
reference's binding `matmul<fn>(A, B)` (bf16_matmul/matmul.cpp:24-42) takes
A [M,K] and B stored [N,K] and returns C = A @ B.T (bf16_matmul/README.md:7,
bf16_matmul/main.py:29-42).  Unlike the reference it reads N from B.size(0)
(the reference takes B.size(1), matmul.cpp:29, which is only right for square
shapes), checks dtype/device/layout, and runs on torch's current stream.

`gemm(A, B, b_layout=...)` is the general entry: b_layout "nk" is the
reference's layout, "kn" is B stored [K,N] row-major (C = A @ B).

Every call goes through the C ABI (include/b200_gemm.h); there is no CPU or
library fallback.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import B200GemmError

_LAYOUTS = {"nk": _lib.B200_B_NK, "kn": _lib.B200_B_KN}


def _check_operand(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dim() != 2:
        raise ValueError(f"{name} must be 2-D, got shape {tuple(t.shape)}")
    if t.stride(1) != 1 and t.numel() > 0:
        raise ValueError(f"{name} must be row-major (stride(1) == 1), got strides {t.stride()}")


def gemm(a: torch.Tensor, b: torch.Tensor, *, b_layout: str = "nk", out: torch.Tensor | None = None,
         stream: torch.cuda.Stream | None = None, split_k: bool = False, alpha: float = 1.0, beta: float = 0.0,
         c: torch.Tensor | None = None, bias: torch.Tensor | None = None,
         out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """C = A @ op(B) in bf16 with fp32 accumulation on a B200 (sm_100a).

    Fused epilogue (b200_gemm_bf16_ex): with any of alpha != 1, beta != 0
    (c: bf16 [M, N], may be `out` itself), bias (bf16 [N]) or
    out_dtype=torch.float32 the result is
        out = alpha * (A @ op(B)) + bias + beta * c
    computed in fp32 from the accumulator, in that order, and written once as
    out_dtype (bf16 or fp32).

    split_k=True lets the tiles of the last, partial wave be split along K
    across CTA pairs (b200_gemm_bf16_ws), which shortens that wave.  It changes
    the fp32 summation order of those tiles: results stay within the bf16
    tolerance of the exact product but are no longer bit-identical to a
    sequential-K GEMM such as cuBLAS (near-zero outputs can differ by more than
    torch.testing.assert_close's default atol).  The default keeps the
    sequential K order of the reference kernels."""
    if b_layout not in _LAYOUTS:
        raise ValueError(f"b_layout must be 'nk' or 'kn', got {b_layout!r}")
    _check_operand("A", a)
    _check_operand("B", b)
    if a.device != b.device:
        raise ValueError("A and B must be on the same device")
    M, K = a.shape
    if b_layout == "nk":
        N, Kb = b.shape
    else:
        Kb, N = b.shape
    if Kb != K:
        raise ValueError(f"inner dimensions differ: A is {tuple(a.shape)}, B ({b_layout}) is {tuple(b.shape)}")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"out_dtype must be torch.bfloat16 or torch.float32, got {out_dtype}")
    fused = alpha != 1.0 or beta != 0.0 or bias is not None or out_dtype == torch.float32
    if fused and split_k:
        raise ValueError("split_k is not available with a fused epilogue")
    if beta != 0.0:
        if c is None:
            raise ValueError("beta != 0 needs c")
        _check_operand("c", c)
        if tuple(c.shape) != (M, N) or c.device != a.device:
            raise ValueError(f"c must be a [{M}, {N}] tensor on the device of A")
    if bias is not None:
        if not isinstance(bias, torch.Tensor) or bias.dtype != torch.bfloat16 or bias.device != a.device \
                or tuple(bias.shape) != (N,) or (N > 1 and bias.stride(0) != 1):
            raise ValueError(f"bias must be a contiguous bf16 [{N}] tensor on the device of A")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    else:
        if out.dtype != out_dtype:
            raise TypeError(f"out must be {out_dtype}, got {out.dtype}")
        if out.dtype == torch.bfloat16:
            _check_operand("out", out)
        elif not out.is_cuda or out.dim() != 2 or (out.stride(1) != 1 and out.numel() > 0):
            raise ValueError("out must be a row-major 2-D CUDA tensor")
        if tuple(out.shape) != (M, N):
            raise ValueError(f"out must have shape {(M, N)}, got {tuple(out.shape)}")
        if out.device != a.device:
            raise ValueError("out must be on the same device as A")
    lib = _lib.load()
    layout = _LAYOUTS[b_layout]
    dev_index = a.device.index
    switch = dev_index != torch.cuda.current_device()
    if switch:
        prev = torch.cuda.current_device()
        torch.cuda.set_device(dev_index)
    try:
        s = stream if stream is not None else torch.cuda.current_stream(a.device)
        if fused:
            epi = _lib.Epilogue(alpha=float(alpha), beta=float(beta),
                                c_in=c.data_ptr() if beta != 0.0 else None,
                                ldc_in=max(c.stride(0), 1) if beta != 0.0 else 0,
                                bias=bias.data_ptr() if bias is not None else None,
                                d_dtype=_lib.B200_DTYPE_F32 if out_dtype == torch.float32 else _lib.B200_DTYPE_BF16)
            rc = lib.b200_gemm_bf16_ex(
                ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                M, N, K, max(a.stride(0), 1), max(b.stride(0), 1), max(out.stride(0), 1),
                layout, ctypes.byref(epi), ctypes.c_void_p(s.cuda_stream))
            if rc != _lib.B200_OK:
                raise B200GemmError(rc, f"M={M} N={N} K={K} b_layout={b_layout} (fused epilogue)")
            return out
        # Split-K workspace for the last wave of tiles (0 bytes when the shape
        # does not need it); torch's caching allocator makes this cheap and
        # stream-safe, so concurrent calls never share a workspace.
        ws_bytes = workspace_bytes(M, N, K, b_layout) if split_k else 0
        ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=a.device) if ws_bytes else None
        if ws is not None and stream is not None:
            ws.record_stream(s)  # allocated on the current stream, used on `s`
        ws_ptr = ((ws.data_ptr() + 255) // 256 * 256) if ws is not None else None
        rc = lib.b200_gemm_bf16_ws(
            ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(out.data_ptr()),
            M, N, K,
            max(a.stride(0), 1), max(b.stride(0), 1), max(out.stride(0), 1),
            layout, ctypes.c_void_p(ws_ptr), ws_bytes, ctypes.c_void_p(s.cuda_stream))
    finally:
        if switch:
            torch.cuda.set_device(prev)
    if rc != _lib.B200_OK:
        raise B200GemmError(rc, f"M={M} N={N} K={K} b_layout={b_layout}")
    return out


def gemm_f32(a: torch.Tensor, b: torch.Tensor, *, b_layout: str = "kn", out: torch.Tensor | None = None,
             stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """fp32 C = A @ op(B) for fp32 A, B (the reference's fp32_matmul operator; its B is [K,N],
    b_layout "kn"), on the bf16 tensor cores through an exact three-way bf16 split of each
    operand (b200_gemm_f32); the split operands go to a workspace from torch's allocator."""
    if b_layout not in _LAYOUTS:
        raise ValueError(f"b_layout must be 'nk' or 'kn', got {b_layout!r}")
    for name, t in (("A", a), ("B", b)):
        if not isinstance(t, torch.Tensor) or t.dtype != torch.float32:
            raise TypeError(f"{name} must be a float32 tensor")
        if not t.is_cuda or t.dim() != 2 or (t.numel() > 0 and t.stride(1) != 1):
            raise ValueError(f"{name} must be a row-major 2-D CUDA tensor")
    if a.device != b.device:
        raise ValueError("A and B must be on the same device")
    M, K = a.shape
    N, Kb = (b.shape[0], b.shape[1]) if b_layout == "nk" else (b.shape[1], b.shape[0])
    if Kb != K:
        raise ValueError(f"inner dimensions differ: A is {tuple(a.shape)}, B ({b_layout}) is {tuple(b.shape)}")
    if out is None:
        # D is written by TMA: its row pitch must be a multiple of 4 floats.
        out = torch.empty((M, (N + 3) // 4 * 4), dtype=torch.float32, device=a.device)[:, :N]
    elif out.dtype != torch.float32 or tuple(out.shape) != (M, N) or out.device != a.device \
            or (out.numel() > 0 and out.stride(1) != 1):
        raise ValueError(f"out must be a row-major float32 [{M}, {N}] tensor on the device of A")
    lib = _lib.load()
    layout = _LAYOUTS[b_layout]
    with torch.cuda.device(a.device):
        s = stream if stream is not None else torch.cuda.current_stream(a.device)
        n = ctypes.c_size_t(0)
        rc = lib.b200_gemm_f32_workspace_bytes(M, N, K, layout, ctypes.byref(n))
        if rc != _lib.B200_OK:
            raise B200GemmError(rc)
        ws = torch.empty(n.value + 256, dtype=torch.uint8, device=a.device) if n.value else None
        if ws is not None and stream is not None:
            ws.record_stream(s)
        ws_ptr = ((ws.data_ptr() + 255) // 256 * 256) if ws is not None else None
        rc = lib.b200_gemm_f32(ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()),
                               ctypes.c_void_p(out.data_ptr()), M, N, K, max(a.stride(0), 1), max(b.stride(0), 1),
                               max(out.stride(0), 1), layout, ctypes.c_void_p(ws_ptr), n.value,
                               ctypes.c_void_p(s.cuda_stream))
    if rc != _lib.B200_OK:
        raise B200GemmError(rc, f"fp32 M={M} N={N} K={K} b_layout={b_layout}")
    return out


def flash_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, causal: bool = True,
               out: torch.Tensor | None = None, stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """O = softmax(Q K^T / sqrt(D)) V (the reference's flash_attn operator, flash_attn/flash_attn.cpp:16-25),
    through b200_flash_attn_bf16.  Q is [batch, seq, heads, 128] bf16; K and V are [batch, seq, kv_heads, 128]
    with heads a multiple of kv_heads (grouped-query attention: query head h uses key/value head
    h // (heads // kv_heads), as fa2_tma_lazy_rescale.cu:113-114)."""
    for name, t in (("Q", q), ("K", k), ("V", v)):
        if not isinstance(t, torch.Tensor) or t.dtype != torch.bfloat16 or not t.is_cuda or t.dim() != 4:
            raise ValueError(f"{name} must be a 4-D bfloat16 CUDA tensor [batch, seq, heads, head_dim]")
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    B, S, H, D = q.shape
    Hkv = k.shape[2]
    if k.shape != (B, S, Hkv, D) or v.shape != k.shape or k.device != q.device or v.device != q.device:
        raise ValueError("K and V must have Q's batch, seq and head_dim, the same shape, and Q's device")
    if Hkv == 0 and H != 0 or Hkv != 0 and H % Hkv != 0:
        raise ValueError(f"the number of query heads ({H}) must be a multiple of the key/value heads ({Hkv})")
    if out is None:
        out = torch.empty_like(q)
    elif out.shape != q.shape or out.dtype != torch.bfloat16 or not out.is_contiguous() or out.device != q.device:
        raise ValueError("out must be a contiguous bfloat16 tensor shaped like Q")
    lib = _lib.load()
    with torch.cuda.device(q.device):
        s = stream if stream is not None else torch.cuda.current_stream(q.device)
        rc = lib.b200_flash_attn_bf16(ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(k.data_ptr()),
                                      ctypes.c_void_p(v.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                      B, S, H, Hkv, D, 1 if causal else 0, ctypes.c_void_p(s.cuda_stream))
    if rc != _lib.B200_OK:
        raise B200GemmError(rc, f"flash_attn B={B} S={S} H={H} Hkv={Hkv} D={D}")
    return out


def workspace_bytes(M: int, N: int, K: int, b_layout: str = "nk") -> int:
    """Split-K workspace (bytes) b200_gemm_bf16_ws wants for this shape on the current device."""
    n = ctypes.c_size_t(0)
    rc = _lib.load().b200_gemm_workspace_bytes(M, N, K, _LAYOUTS[b_layout], ctypes.byref(n))
    if rc != _lib.B200_OK:
        raise B200GemmError(rc)
    return n.value


def matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Reference-compatible operator: B is [N,K], returns A @ B.T (bf16_matmul/matmul.cpp:24-42)."""
    return gemm(a, b, b_layout="nk")


def check_status(stream: torch.cuda.Stream | None = None, device: torch.device | int | None = None) -> int:
    """Synchronise and read/clear the device status word; raises B200GemmError on a device timeout."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        s = stream if stream is not None else torch.cuda.current_stream(dev)
        bits = ctypes.c_uint32(0)
        rc = lib.b200_gemm_status(ctypes.c_void_p(s.cuda_stream), ctypes.byref(bits))
    if rc != _lib.B200_OK:
        raise B200GemmError(rc, f"device status bits 0x{bits.value:x}")
    return bits.value


def set_timeout_ns(ns: int, device: torch.device | int | None = None) -> None:
    """Time limit for every device-side wait of later launches on `device` (0 = default 4 s)."""
    lib = _lib.load()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        rc = lib.b200_gemm_set_timeout_ns(int(ns))
    if rc != _lib.B200_OK:
        raise B200GemmError(rc)


_KERNELS = {"auto": _lib.B200_KERNEL_AUTO, "single": _lib.B200_KERNEL_SINGLE, "pair": _lib.B200_KERNEL_PAIR,
            "skinny": _lib.B200_KERNEL_SKINNY}


def set_kernel(which: str) -> None:
    """Force a kernel for later calls ("auto", "single", "pair", "skinny"); for tests and tuning."""
    if which not in _KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}")
    rc = _lib.load().b200_gemm_set_kernel(_KERNELS[which])
    if rc != _lib.B200_OK:
        raise B200GemmError(rc)


_ATTN_KERNELS = {"auto": _lib.B200_ATTN_KERNEL_AUTO, "single": _lib.B200_ATTN_KERNEL_SINGLE,
                 "pair": _lib.B200_ATTN_KERNEL_PAIR}


def flash_attn_set_kernel(which: str) -> None:
    """Force the attention kernel for later flash_attn calls ("auto", "single": one CTA per two query
    tiles, "pair": a CTA pair per four); for tests and tuning, every choice computes the same result."""
    if which not in _ATTN_KERNELS:
        raise ValueError(f"attention kernel must be one of {sorted(_ATTN_KERNELS)}")
    rc = _lib.load().b200_flash_attn_set_kernel(_ATTN_KERNELS[which])
    if rc != _lib.B200_OK:
        raise B200GemmError(rc)

