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
import os

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


GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", ["f32_37x53x301", "f32_128x128x256", "f32_256x128x96"])
def test_f32_vs_reference_golden(name):
    """Against the reference's own fp32 kernel outputs (v1, run on a B200 by
    tests/golden/make_golden_f32.py): as accurate as they are, by the bar above."""
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    a, b = d["A"], d["B"]
    c = b200_gemm.gemm_f32(torch.from_numpy(a).to(DEV), torch.from_numpy(b).to(DEV), b_layout="kn")
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    exact, _ = o.gemm_f32_f64(a, b, 1)
    ours, ref = _errors(c.cpu().numpy(), exact), _errors(d["C_ref_v1"], exact)
    ctx = f"{name}: ours {ours}, reference v1 {ref}"
    assert ours[0] <= 4.0 * ref[0] and ours[1] <= 5.0 * ref[1] and ours[1] < 1e-5, ctx


def test_f32_vs_reference_live():
    """Against the reference's fp32 kernels run live (oracle/_ref/libref_f32.so) on
    its benchmark layout at 512 x 1024 x 768: v1 and its best kernel, v5."""
    if not o.ref_f32_available():
        pytest.skip("oracle/_ref/libref_f32.so not built (needs the reference sources)")
    lib = o.ref_f32_lib()
    M, N, K = 512, 1024, 768
    g = torch.Generator().manual_seed(5)
    a, b = torch.randn((M, K), generator=g).to(DEV), torch.randn((K, N), generator=g).to(DEV)
    ours = b200_gemm.gemm_f32(a, b, b_layout="kn")
    outs = {}
    for v, f in (("v1", lib.ref_matmul_f32_v1), ("v5", lib.ref_matmul_f32_v5)):
        c = torch.empty((M, N), device=DEV)
        torch.cuda.synchronize()
        assert f(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K) == 0
        torch.cuda.synchronize()
        outs[v] = c.cpu().numpy()
    assert b200_gemm.check_status() == 0
    exact, _ = o.gemm_f32_f64(a.cpu().numpy(), b.cpu().numpy(), 1)
    e = _errors(ours.cpu().numpy(), exact)
    # The CPU restatement is the reference's v1 bit for bit.
    assert np.array_equal(outs["v1"], o.gemm_f32(a.cpu().numpy(), b.cpu().numpy(), 1))
    for v in ("v1", "v5"):
        r = _errors(outs[v], exact)
        assert e[0] <= 4.0 * r[0] and e[1] <= 5.0 * r[1], f"ours {e} vs reference {v} {r}"
