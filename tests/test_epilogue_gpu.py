"""GPU parity tests of the fused epilogue, b200_gemm_bf16_ex (called through
the C ABI by b200_gemm.gemm with alpha / beta / c / bias / out_dtype):

    D = alpha * (A @ op(B)) + bias[n] + beta * C_in[m, n],  bf16 or fp32 D

on every kernel path (skinny without and with cluster split-K, CTA pairs with
256- and 512-column tiles, the single-CTA kernel), both B layouts, ragged
shapes and the in-place form (C_in = D).  The truth is the CPU oracle's
restatement (oracle.epilogue) applied to the fp64 product; bf16 results are
held to the same bounds as the plain GEMM (tests/_util.check_parity), fp32
results to 2^-12 of max(|exact|, rms) — 8x finer than one bf16 ulp.
"""
import numpy as np
import pytest
import torch

import b200_gemm
from oracle import oracle as o
from tests._util import bits, check_parity, uniform_bf16

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _pad(x: int, m: int) -> int:
    return max((x + m - 1) // m * m, m)


def _dev2d(t: torch.Tensor, mult: int = 8) -> torch.Tensor:
    """Device copy with the row pitch rounded up to `mult` elements."""
    r, c = t.shape
    buf = torch.zeros((r, _pad(c, mult)), dtype=t.dtype, device=DEV)
    buf[:, :c] = t.to(DEV)
    return buf[:, :c]


CASES = [  # name, M, N, K, forced kernel
    ("skinny_s1", 40, 19000, 256, "auto"),      # 149 tiles: no split
    ("skinny_s8", 100, 1000, 3000, "auto"),     # 8 tiles x 8 splits
    ("skinny_s2", 16, 5000, 1000, "auto"),      # 40 tiles x 2 splits
    ("pair_wide", 4096, 4096, 128, "auto"),     # 256 x 512 pair tiles (rows sampled for the oracle)
    ("pair_ragged", 1000, 2601, 520, "auto"),   # 256 x 256 pair tiles, N ragged
    ("pair_forced", 300, 520, 200, "pair"),
    ("single_forced", 300, 520, 200, "single"),
]
EPIS = {
    "alpha_bias": dict(alpha=0.5, bias=True),
    "residual": dict(beta=1.0),
    "f32_out": dict(f32=True),
    "all_f32": dict(alpha=1.25, beta=-0.75, bias=True, f32=True),
    "in_place": dict(beta=1.0, bias=True, inplace=True),
}


@pytest.fixture
def kernel():
    yield b200_gemm.set_kernel
    b200_gemm.set_kernel("auto")


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("epi_name", list(EPIS))
@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_fused_epilogue_vs_oracle(case, epi_name, layout, kernel):
    name, M, N, K, forced = case
    e = EPIS[epi_name]
    kernel(forced)
    seed = M + 3 * N + 7 * K + len(epi_name)
    a = uniform_bf16((M, K), seed)
    b_nk = uniform_bf16((N, K), seed + 1)
    b = b_nk if layout == "nk" else b_nk.t().contiguous()
    alpha, beta = e.get("alpha", 1.0), e.get("beta", 0.0)
    bias = uniform_bf16((N,), seed + 2) if e.get("bias") else None
    c_in = uniform_bf16((M, N), seed + 3) if beta != 0.0 else None
    f32 = e.get("f32", False)
    out_dtype = torch.float32 if f32 else torch.bfloat16

    ad, bd = _dev2d(a), _dev2d(b)
    if e.get("inplace"):
        out = _dev2d(c_in)
        cd = out
    else:
        out = _dev2d(torch.full((M, N), float("nan"), dtype=out_dtype), 4 if f32 else 8)
        cd = _dev2d(c_in) if c_in is not None else None
    biasd = bias.to(DEV) if bias is not None else None
    res = b200_gemm.gemm(ad, bd, b_layout=layout, out=out, alpha=alpha, beta=beta, c=cd, bias=biasd,
                         out_dtype=out_dtype)
    assert res.data_ptr() == out.data_ptr()
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0

    rows = np.arange(M) if M <= 1024 else np.array(sorted({0, M - 1, *range(5, M, M // 67)}))
    a_r = bits(a)[rows]
    c_r = bits(c_in)[rows] if c_in is not None else None
    bias_b = bits(bias) if bias is not None else None
    exact = o.epilogue(o.gemm_f64(a_r, bits(b_nk), 0)[0], alpha, beta, c_r, bias_b)
    acc32 = o.gemm_f32acc(a_r, bits(b_nk), 0)
    ctx = f"{name} {epi_name} {layout}"
    if not f32:
        check_parity(bits(res)[rows], exact, o.epilogue(acc32, alpha, beta, c_r, bias_b, out="bf16"), ctx=ctx)
    else:
        got = res.cpu().numpy()[rows].astype(np.float64)
        assert np.all(np.isfinite(got)), f"{ctx}: non-finite output"
        rms = float(np.sqrt(np.mean(exact ** 2)))
        tol = 2.0 ** -12 * np.maximum(np.abs(exact), rms)
        assert np.all(np.abs(got - exact) <= tol), f"{ctx}: max |dD| / tol = {np.max(np.abs(got - exact) / tol):.3f}"
        orc = o.epilogue(acc32, alpha, beta, c_r, bias_b, out="f32").astype(np.float64)
        assert np.all(np.abs(got - orc) <= tol), f"{ctx}: fp32 D differs from the oracle's fp32 epilogue"
        # fp32 really kept: most values are not bf16 numbers.
        low = (res.cpu().numpy()[rows].view(np.uint32) & 0xFFFF) != 0
        assert np.mean(low) > 0.5, f"{ctx}: fp32 output looks rounded to bf16"


def test_epilogue_argument_errors():
    a = torch.zeros((64, 64), dtype=torch.bfloat16, device=DEV)
    b = torch.zeros((64, 64), dtype=torch.bfloat16, device=DEV)
    c = torch.zeros((64, 64), dtype=torch.bfloat16, device=DEV)
    bias = torch.zeros((64,), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        b200_gemm.gemm(a, b, beta=1.0)  # beta without c
    with pytest.raises(ValueError):
        b200_gemm.gemm(a, b, bias=bias[:32])  # wrong bias length
    with pytest.raises(ValueError):
        b200_gemm.gemm(a, b, bias=bias, split_k=True)
    with pytest.raises(b200_gemm.B200GemmError):
        b200_gemm.gemm(a[:, :0], b[:, :0], bias=bias)  # K = 0 with an epilogue
    out32 = torch.zeros((64, 64), dtype=torch.float32, device=DEV)
    from b200_gemm import _lib
    import ctypes
    lib = _lib.load()
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # C_in may alias D only when D is bf16 with the same pitch.
    epi = _lib.Epilogue(alpha=1.0, beta=1.0, c_in=out32.data_ptr(), ldc_in=64, bias=None, d_dtype=_lib.B200_DTYPE_F32)
    rc = lib.b200_gemm_bf16_ex(a.data_ptr(), b.data_ptr(), out32.data_ptr(), 64, 64, 64, 64, 64, 64, 0,
                               ctypes.byref(epi), s)
    assert rc == _lib.B200_ERR_INVALID_ARG
    # Misaligned bias.
    epi = _lib.Epilogue(alpha=1.0, beta=0.0, c_in=None, ldc_in=0, bias=bias.data_ptr() + 2,
                        d_dtype=_lib.B200_DTYPE_BF16)
    rc = lib.b200_gemm_bf16_ex(a.data_ptr(), b.data_ptr(), c.data_ptr(), 64, 64, 64, 64, 64, 64, 0,
                               ctypes.byref(epi), s)
    assert rc == _lib.B200_ERR_ALIGNMENT
    # epi == NULL is the plain GEMM.
    rc = lib.b200_gemm_bf16_ex(a.data_ptr(), b.data_ptr(), c.data_ptr(), 64, 64, 64, 64, 64, 64, 0, None, s)
    assert rc == _lib.B200_OK
    torch.cuda.synchronize()


@pytest.mark.parametrize("ldd", [64, 72])
def test_k_zero_fp32_d_is_zero_filled(ldd):
    """K = 0 with fp32 D and no other epilogue term: D = 0 over its whole
    [M, N] extent, with D's own 4-byte elements and row pitch (a bf16-sized
    fill would clear half of each row and the wrong rows); the padding
    columns beyond N keep their contents."""
    M, N = 96, 60
    import ctypes
    from b200_gemm import _lib
    lib = _lib.load()
    a = torch.empty((M, 8), dtype=torch.bfloat16, device=DEV)
    b = torch.empty((N, 8), dtype=torch.bfloat16, device=DEV)
    buf = torch.full((M, ldd), 7.0, dtype=torch.float32, device=DEV)
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    epi = _lib.Epilogue(alpha=1.0, beta=0.0, c_in=None, ldc_in=0, bias=None, d_dtype=_lib.B200_DTYPE_F32)
    rc = lib.b200_gemm_bf16_ex(a.data_ptr(), b.data_ptr(), buf.data_ptr(), M, N, 0, 8, 8, ldd, 0,
                               ctypes.byref(epi), s)
    assert rc == _lib.B200_OK
    torch.cuda.synchronize()
    assert torch.count_nonzero(buf[:, :N]) == 0
    assert torch.all(buf[:, N:] == 7.0)
    # the same through the Python API
    out = torch.full((M, N), 5.0, dtype=torch.float32, device=DEV)
    b200_gemm.gemm(a[:, :0], b[:, :0], out=out, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
