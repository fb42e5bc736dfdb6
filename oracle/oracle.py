"""ctypes wrapper of oracle/gemm_oracle.c (CPU restatement of the reference's
BF16 GEMM: bf16 inputs, fp32 accumulation in K=16 partial sums, RN-even bf16
output; see the header of gemm_oracle.c for the reference lines it follows).

TEST INFRASTRUCTURE ONLY — imported by tests/, __graft_entry__.smoke() and
bench.py's CPU baseline, never by the product path.

Arrays are numpy: bf16 values travel as their uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_LIB_PATH = os.path.join(HERE, "_ref", "libref_v8_tuned.so")
REF_F32_LIB_PATH = os.path.join(HERE, "_ref", "libref_f32.so")

_lib = None
_ref = None


def build() -> None:
    """Compile the C oracle (gcc) and, when the reference checkout is present, oracle/_ref."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)
    from oracle import build_ref_fa2  # the reference's attention operator, when its sources are present

    build_ref_fa2.build()


def _load():
    global _lib
    if _lib is None:
        src = os.path.join(HERE, "gemm_oracle.c")
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            subprocess.run(["make", "-s", "-C", HERE], check=True)
        lib = ctypes.CDLL(LIB_PATH)
        i64 = ctypes.c_int64
        vp = ctypes.c_void_p
        lib.oracle_gemm_bf16_f32acc.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int]
        lib.oracle_gemm_bf16.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int]
        lib.oracle_gemm_bf16_f64.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int]
        lib.oracle_gemm_f32.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int]
        lib.oracle_gemm_f32_f64.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, ctypes.c_int, ctypes.c_int]
        lib.oracle_gemm_f32.restype = ctypes.c_int
        lib.oracle_gemm_f32_f64.restype = ctypes.c_int
        lib.oracle_f32_to_bf16.argtypes = [vp, vp, i64]
        lib.oracle_bf16_to_f32.argtypes = [vp, vp, i64]
        for f in (lib.oracle_gemm_bf16_f32acc, lib.oracle_gemm_bf16, lib.oracle_gemm_bf16_f64):
            f.restype = ctypes.c_int
        lib.oracle_num_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def _u16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    if x.dtype != np.uint16:
        raise TypeError(f"expected uint16 bf16 bit patterns, got {x.dtype}")
    return x


def _dims(a: np.ndarray, b: np.ndarray, b_layout: int):
    M, K = a.shape
    if b_layout == 0:
        N, Kb = b.shape
    else:
        Kb, N = b.shape
    if Kb != K:
        raise ValueError(f"inner dims differ: {a.shape} vs {b.shape} (layout {b_layout})")
    return M, N, K


def num_threads() -> int:
    return int(_load().oracle_num_threads())


def gemm_f32acc(a: np.ndarray, b: np.ndarray, b_layout: int = 0, threads: int = 0) -> np.ndarray:
    """fp32 result (before bf16 rounding) of A @ op(B); b_layout 0: B is [N,K], 1: B is [K,N]."""
    a, b = _u16(a), _u16(b)
    M, N, K = _dims(a, b, b_layout)
    c = np.empty((M, N), dtype=np.float32)
    rc = _load().oracle_gemm_bf16_f32acc(a.ctypes.data, b.ctypes.data, c.ctypes.data, M, N, K,
                                         max(K, 1), b.shape[1] if b.size else 1, max(N, 1), b_layout, threads)
    if rc != 0:
        raise RuntimeError("oracle_gemm_bf16_f32acc failed")
    return c


def gemm_bf16(a: np.ndarray, b: np.ndarray, b_layout: int = 0, threads: int = 0) -> np.ndarray:
    """bf16 bit patterns of RN(A @ op(B)) with fp32 accumulation — what the reference kernel outputs."""
    a, b = _u16(a), _u16(b)
    M, N, K = _dims(a, b, b_layout)
    c = np.empty((M, N), dtype=np.uint16)
    rc = _load().oracle_gemm_bf16(a.ctypes.data, b.ctypes.data, c.ctypes.data, M, N, K,
                                  max(K, 1), b.shape[1] if b.size else 1, max(N, 1), b_layout, threads)
    if rc != 0:
        raise RuntimeError("oracle_gemm_bf16 failed")
    return c


def gemm_f64(a: np.ndarray, b: np.ndarray, b_layout: int = 0, threads: int = 0):
    """(near-exact fp64 product, fp64 sum of |a*b|) of A @ op(B)."""
    a, b = _u16(a), _u16(b)
    M, N, K = _dims(a, b, b_layout)
    c = np.empty((M, N), dtype=np.float64)
    s = np.empty((M, N), dtype=np.float64)
    rc = _load().oracle_gemm_bf16_f64(a.ctypes.data, b.ctypes.data, c.ctypes.data, s.ctypes.data, M, N, K,
                                      max(K, 1), b.shape[1] if b.size else 1, b_layout, threads)
    if rc != 0:
        raise RuntimeError("oracle_gemm_bf16_f64 failed")
    return c, s


def _f32dims(a: np.ndarray, b: np.ndarray, b_layout: int):
    M, K = a.shape
    N = b.shape[0] if b_layout == 0 else b.shape[1]
    Kb = b.shape[1] if b_layout == 0 else b.shape[0]
    if Kb != K:
        raise ValueError("inner dimensions differ")
    return M, N, K


def gemm_f32(a: np.ndarray, b: np.ndarray, b_layout: int = 1, threads: int = 0) -> np.ndarray:
    """fp32 GEMM as the reference's fp32_matmul kernels compute it (one fp32 FMA chain per output,
    k ascending; fp32_matmul/matmul.cu:18-36).  b_layout 1 = B [K,N] (the reference's), 0 = B [N,K]."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M, N, K = _f32dims(a, b, b_layout)
    c = np.empty((M, N), dtype=np.float32)
    rc = _load().oracle_gemm_f32(a.ctypes.data, b.ctypes.data, c.ctypes.data, M, N, K, max(K, 1),
                                 b.shape[1] if b.size else 1, b_layout, threads)
    if rc != 0:
        raise RuntimeError("oracle_gemm_f32 failed")
    return c


def gemm_f32_f64(a: np.ndarray, b: np.ndarray, b_layout: int = 1, threads: int = 0):
    """(near-exact fp64 product, fp64 sum of |a*b|) of fp32 operands."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    M, N, K = _f32dims(a, b, b_layout)
    c = np.empty((M, N), dtype=np.float64)
    s = np.empty((M, N), dtype=np.float64)
    rc = _load().oracle_gemm_f32_f64(a.ctypes.data, b.ctypes.data, c.ctypes.data, s.ctypes.data, M, N, K,
                                     max(K, 1), b.shape[1] if b.size else 1, b_layout, threads)
    if rc != 0:
        raise RuntimeError("oracle_gemm_f32_f64 failed")
    return c, s


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    _load().oracle_f32_to_bf16(x.ctypes.data, y.ctypes.data, x.size)
    return y


def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    x = _u16(x)
    y = np.empty(x.shape, dtype=np.float32)
    _load().oracle_bf16_to_f32(x.ctypes.data, y.ctypes.data, x.size)
    return y


def epilogue(acc: np.ndarray, alpha: float = 1.0, beta: float = 0.0, c_in: np.ndarray | None = None,
             bias: np.ndarray | None = None, out: str = "bf16") -> np.ndarray:
    """Fused epilogue of b200_gemm_bf16_ex on an fp32 accumulator `acc` [M, N]:
    D = alpha * acc + bias[n] + beta * c_in[m, n], one fp32 operation at a
    time in that order (no fused multiply-add), then RN-even bf16 (uint16
    bits) or fp32.  bias / c_in are bf16 bit patterns.  The reference has no
    epilogue (its kernels store bf16(acc) only, bf16_matmul/matmul_v8_tuned.cu:
    152-178); this restates the documented semantics of the new entry point.
    Also used on the fp64 product (acc float64) for a near-exact reference."""
    ft = np.float64 if acc.dtype == np.float64 else np.float32
    acc = np.asarray(acc, dtype=ft)
    x = (ft(alpha) * acc).astype(ft)
    bvec = bf16_to_f32(bias).astype(ft) if bias is not None else np.zeros(acc.shape[1], dtype=ft)
    x = (x + bvec[None, :]).astype(ft)
    cmat = bf16_to_f32(c_in).astype(ft) if (c_in is not None and beta != 0.0) else np.zeros_like(x)
    x = (x + (ft(beta) * cmat).astype(ft)).astype(ft)
    if out == "f32" or ft == np.float64:
        return x
    return f32_to_bf16(x)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool) -> np.ndarray:
    """Exact (fp64) attention of bf16 inputs given as uint16 bit patterns, Q of shape
    [batch, seq, heads, head_dim], K and V [batch, seq, kv_heads, head_dim]:
    O = softmax(Q K^T / sqrt(D), causal mask) V, the operator the reference's
    flash_attn kernel computes and checks against F.scaled_dot_product_attention
    (flash_attn/main.py:36-47).  Query head h uses key/value head
    h // (heads // kv_heads) (fa2_tma_lazy_rescale.cu:113-114)."""
    def f64(x):
        return bf16_to_f32(np.ascontiguousarray(x)).astype(np.float64)
    qf, kf, vf = f64(q), f64(k), f64(v)
    B, S, H, D = qf.shape
    group = H // kf.shape[2]
    out = np.empty((B, S, H, D), dtype=np.float64)
    mask = np.triu(np.ones((S, S), dtype=bool), 1) if causal else None
    for b in range(B):
        for h in range(H):
            hk = h // group
            s = qf[b, :, h, :] @ kf[b, :, hk, :].T / np.sqrt(D)
            if mask is not None:
                s[mask] = -np.inf
            s = s - s.max(axis=1, keepdims=True)
            p = np.exp(s)
            out[b, :, h, :] = (p / p.sum(axis=1, keepdims=True)) @ vf[b, :, hk, :]
    return out


# --- the reference's own kernel (oracle/_ref), GPU only ---------------------

def ref_available() -> bool:
    return os.path.exists(REF_LIB_PATH)


def ref_lib():
    """ctypes handle of oracle/_ref/libref_v8_tuned.so: the reference's matmul_v8_tuned
    (bf16_matmul/matmul_v8_tuned.cu:215-257) rebuilt for sm_100a."""
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(REF_LIB_PATH)
        lib.ref_matmul_v8_tuned.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                            ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.ref_matmul_v8_tuned.restype = ctypes.c_int
        _ref = lib
    return _ref


_ref_f32 = None


def ref_f32_available() -> bool:
    return os.path.exists(REF_F32_LIB_PATH)


def ref_f32_lib():
    """ctypes handle of oracle/_ref/libref_f32.so: the reference's fp32 kernels
    (fp32_matmul/matmul.cu, v1 :18-36 and v5 :231-325) rebuilt for sm_100a."""
    global _ref_f32
    if _ref_f32 is None:
        lib = ctypes.CDLL(REF_F32_LIB_PATH)
        for f in (lib.ref_matmul_f32_v1, lib.ref_matmul_f32_v5):
            f.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
            f.restype = ctypes.c_int
        _ref_f32 = lib
    return _ref_f32
