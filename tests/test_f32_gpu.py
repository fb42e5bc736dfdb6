"""GPU tests of the fp32 GEMM (b200_gemm_f32: the reference's fp32_matmul
operator on the bf16 tensor cores through an exact three-way bf16 split of
each operand).

The truth is the fp64 product of the fp32 inputs (oracle.gemm_f32_f64).  The
bar is the reference's own fp32 arithmetic, restated on the CPU
(oracle.gemm_f32: one fp32 FMA chain per output, fp32_matmul/matmul.cu:18-36;
cuBLAS's fp32 GEMM gives the same numbers bit for bit): our largest error may
be at most 4x its and our relative Frobenius error at most 5x its (measured
1.3x to 3.9x, growing with K) and below 1e-5.  The factor is the
tensor cores' fp32 accumulation, which over K' = 6K steps is not a
round-to-nearest FMA chain; the errors stay around 1e-6 relative (TF32 would
be ~1e-3, bf16 ~4e-3).
"""
import numpy as np
import pytest
import torch

import b200_gemm
from oracle import oracle as o

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _errors(c: np.ndarray, exact: np.ndarray):
    d = np.abs(c.astype(np.float64) - exact)
    return float(d.max()), float(np.linalg.norm(d) / max(np.linalg.norm(exact), 1e-300))


@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("shape", [(256, 384, 320), (129, 257, 1000), (64, 5000, 2000), (1000, 2600, 520),
                                   (4096, 4096, 4096)], ids=lambda s: "x".join(map(str, s)))
def test_f32_gemm_as_accurate_as_fp32(shape, layout):
    M, N, K = shape
    g = torch.Generator().manual_seed(M + N + K)
    a = torch.randn((M, K), generator=g)
    b_kn = torch.randn((K, N), generator=g)
    b = b_kn if layout == "kn" else b_kn.t().contiguous()
    c = b200_gemm.gemm_f32(a.to(DEV), b.to(DEV), b_layout=layout)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        c_cublas = torch.matmul(a.to(DEV), b_kn.to(DEV))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    rows = np.arange(M) if M <= 1024 else np.array(sorted({0, M - 1, *range(3, M, M // 53)}))
    a_r = a.numpy()[rows]
    exact, _ = o.gemm_f32_f64(a_r, b_kn.numpy(), 1)
    ours = _errors(c.cpu().numpy()[rows], exact)
    ref = _errors(o.gemm_f32(a_r, b_kn.numpy(), 1), exact)
    cub = _errors(c_cublas.cpu().numpy()[rows], exact)
    ctx = f"{shape} {layout}: max/rel-Frobenius error ours {ours}, fp32 reference {ref}, cuBLAS fp32 {cub}"
    print(ctx)
    assert np.all(np.isfinite(c.cpu().numpy())), ctx
    assert ours[0] <= 4.0 * ref[0], ctx
    assert ours[1] <= 5.0 * ref[1], ctx
    assert ours[1] < 1e-5, ctx


def test_f32_split_is_exact_over_the_exponent_range():
    # Products of values spanning many binades, and exact small-integer cases.
    a = torch.tensor([[1.0, 2.0 ** 20, 3.0e-20, -7.25], [1.0 / 3.0, -1e10, 5e-5, 1.0]], dtype=torch.float32)
    b = torch.tensor([[1.0], [2.0 ** -20], [1.0e20], [4.0]], dtype=torch.float32)
    c = b200_gemm.gemm_f32(a.to(DEV), b.to(DEV), b_layout="kn").cpu().numpy()
    exact, _ = o.gemm_f32_f64(a.numpy(), b.numpy(), 1)
    assert np.allclose(c, exact, rtol=2 ** -22, atol=0), (c, exact)


def test_f32_torch_binding_matches():
    from b200_gemm.binding import load_binding
    module = load_binding()
    g = torch.Generator().manual_seed(5)
    a = torch.randn((300, 200), generator=g).to(DEV)
    b = torch.randn((200, 500), generator=g).to(DEV)
    c1 = module.matmul_b200_f32(a, b)
    c2 = b200_gemm.gemm_f32(a, b)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
    with pytest.raises(ValueError):
        module.matmul_b200_f32(a.to(torch.bfloat16), b)


def test_f32_k_zero_and_empty():
    a = torch.zeros((5, 0), device=DEV)
    b = torch.zeros((0, 7), device=DEV)
    out = torch.full((5, 8), float("nan"), device=DEV)[:, :7]  # D's pitch: a multiple of 4 floats
    c = b200_gemm.gemm_f32(a, b, out=out)
    torch.cuda.synchronize()
    assert torch.equal(c, torch.zeros((5, 7), device=DEV))
    assert b200_gemm.gemm_f32(torch.zeros((0, 4), device=DEV), torch.zeros((4, 3), device=DEV)).shape == (0, 3)
