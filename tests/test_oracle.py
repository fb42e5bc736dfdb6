"""CPU tests of the oracle (gemm_oracle.c): rounding known answers, internal
consistency, accuracy against an fp64 product, and the pin against outputs
of the reference's own kernel (tests/golden/)."""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as o
from tests._util import bf16_bits_to_f64, check_parity

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_bf16_rounding_known_answers():
    # Values chosen on and around bf16 rounding boundaries (8 significant bits).
    x = np.array([1.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8, 1.0 + 2 ** -8 + 2 ** -20, -1.0 - 2 ** -8,
                  3.0e38, 0.0, -0.0, 2 ** -130, np.inf, -np.inf], dtype=np.float32)
    want = np.array([0x3F80, 0x3F80, 0x3F82, 0x3F81, 0xBF80, 0x7F62, 0x0000, 0x8000, 0x0008, 0x7F80, 0xFF80],
                    dtype=np.uint16)
    got = o.f32_to_bf16(x)
    assert np.array_equal(got, want), [hex(v) for v in got]
    assert o.f32_to_bf16(np.array([np.nan], dtype=np.float32))[0] == 0x7FFF
    back = o.bf16_to_f32(want[:5])
    assert back.tolist() == [1.0, 1.0, 1.0 + 2 ** -6, 1.0 + 2 ** -7, -1.0]


def test_epilogue_known_answers():
    # D = alpha * acc + bias + beta * c_in, one fp32 operation at a time.
    acc = np.array([[1.5, -0.0, 3.0, 1.0]], dtype=np.float32)
    bias = o.f32_to_bf16(np.array([0.25, 0.0, -1.0, 2 ** -8], dtype=np.float32))
    c_in = o.f32_to_bf16(np.array([[1.0, 2.0, 0.5, 0.0]], dtype=np.float32))
    got = o.epilogue(acc, 2.0, 0.5, c_in, bias)
    # 2*1.5+0.25+0.5 = 3.75; -0+0+1 = 1; 6-1+0.25 = 5.25; 2+2^-8 -> RN-even tie down to 2.0
    assert [hex(v) for v in got.ravel()] == ["0x4070", "0x3f80", "0x40a8", "0x4000"]
    f = o.epilogue(acc, 2.0, 0.5, c_in, bias, out="f32")
    assert f.dtype == np.float32 and f.ravel().tolist() == [3.75, 1.0, 5.25, 2.0 + 2 ** -8]
    # no bias, beta = 0: only the scale; c_in is not read
    assert o.epilogue(acc, 0.5, 0.0, None, None, out="f32").ravel().tolist() == [0.75, 0.0, 1.5, 0.5]


def test_f32_gemm_known_answers_and_accuracy():
    a = np.array([[1, 2, 3], [-1, 0.5, 4]], dtype=np.float32)
    b = np.array([[1, 2], [1, -1], [1, 0.25]], dtype=np.float32)  # [K,N]
    assert o.gemm_f32(a, b, 1).tolist() == [[6.0, 0.75], [3.5, -1.5]]
    assert o.gemm_f32(a, b.T.copy(), 0).tolist() == [[6.0, 0.75], [3.5, -1.5]]
    rng = np.random.default_rng(3)
    a = rng.standard_normal((40, 700)).astype(np.float32)
    b = rng.standard_normal((700, 30)).astype(np.float32)
    exact, absc = o.gemm_f32_f64(a, b, 1)
    c = o.gemm_f32(a, b, 1).astype(np.float64)
    # fp32 FMA chain: error below K * 2^-24 * sum|a*b| (the classical bound)
    assert np.all(np.abs(c - exact) <= 700 * 2.0 ** -24 * absc)


def test_attention_known_answers():
    # Q = 0: every score is equal, so each row of O is the mean of the values
    # it may see (all of them, or the prefix with a causal mask).
    S, D = 5, 128
    v = np.arange(S * D, dtype=np.float32).reshape(1, S, 1, D) / 64.0
    z = o.f32_to_bf16(np.zeros((1, S, 1, D), dtype=np.float32))
    vb = o.f32_to_bf16(v)
    vv = o.bf16_to_f32(vb).astype(np.float64)[0, :, 0, :]
    full = o.attention(z, z, vb, causal=False)[0, :, 0, :]
    causal = o.attention(z, z, vb, causal=True)[0, :, 0, :]
    assert np.allclose(full, np.broadcast_to(vv.mean(axis=0), (S, D)))
    assert np.allclose(causal, np.cumsum(vv, axis=0) / np.arange(1, S + 1)[:, None])


@pytest.mark.parametrize("name", ["fa2_1x128x2_mha", "fa2_1x192x4_gqa2", "fa2_2x256x2_mha"])
def test_attention_oracle_pinned_to_reference_kernel(name):
    """The exact attention oracle against the reference's own operator
    (fa2_tma_lazy_rescale, causal, run on a B200 by tests/golden/make_golden_attn.py):
    within the reference's check (assert_close rtol = atol = 1e-2,
    flash_attn/main.py:46) and, on average, within a fraction of one bf16 ulp."""
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    exact = o.attention(d["Q"], d["K"], d["V"], True)
    ref = o.bf16_to_f32(d["O_ref_fa2"]).astype(np.float64)
    err = np.abs(ref - exact)
    assert np.all(err <= 1e-2 + 1e-2 * np.abs(exact)), f"{name}: max {err.max():.4f}"
    assert err.mean() < 1e-3, f"{name}: mean {err.mean():.5f}"
    # Rounding the exact result to bf16 reproduces most of the reference's bits.
    same = np.mean(o.f32_to_bf16(exact.astype(np.float32)) == d["O_ref_fa2"])
    assert same > 0.6, f"{name}: only {same:.2%} of elements equal"


@pytest.mark.parametrize("name", ["f32_37x53x301", "f32_128x128x256", "f32_256x128x96"])
def test_f32_oracle_pinned_to_reference_kernel(name):
    """The fp32 restatement reproduces, bit for bit, the reference's fp32 v1 kernel
    (one fp32 multiply-add chain per output over k in order, fp32_matmul/matmul.cu:18-36)
    as run on a B200 by tests/golden/make_golden_f32.py; the reference's v5 and
    cuBLAS agree with it within the classical fp32 dot-product bound."""
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    a, b = d["A"], d["B"]
    c = o.gemm_f32(a, b, 1)
    assert np.array_equal(c.view(np.uint32), d["C_ref_v1"].view(np.uint32)), \
        f"{name}: {np.mean(c != d['C_ref_v1']):.3%} of elements differ from the reference's v1"
    exact, absc = o.gemm_f32_f64(a, b, 1)
    bound = a.shape[1] * 2.0 ** -24 * absc
    for key in ("C_cublas", "C_ref_v5"):
        if key in d.files:
            assert np.all(np.abs(d[key].astype(np.float64) - exact) <= bound), f"{name}: {key} outside the bound"


def test_attention_grouped_heads_match_repeated_heads():
    # heads = 4, kv_heads = 2: query heads 0, 1 use key/value head 0 and 2, 3 use
    # head 1 (fa2_tma_lazy_rescale.cu:113-114), i.e. plain attention with each
    # key/value head repeated twice.
    rng = np.random.default_rng(3)
    q = o.f32_to_bf16(rng.standard_normal((2, 9, 4, 128)).astype(np.float32))
    k = o.f32_to_bf16(rng.standard_normal((2, 9, 2, 128)).astype(np.float32))
    v = o.f32_to_bf16(rng.standard_normal((2, 9, 2, 128)).astype(np.float32))
    for causal in (False, True):
        g = o.attention(q, k, v, causal)
        r = o.attention(q, np.repeat(k, 2, axis=2), np.repeat(v, 2, axis=2), causal)
        assert np.array_equal(g, r)


def test_tiny_known_product():
    # 2x3 @ (2x3)^T with exactly representable values.
    a = o.f32_to_bf16(np.array([[1, 2, 3], [-1, 0.5, 4]], dtype=np.float32))
    b = o.f32_to_bf16(np.array([[1, 1, 1], [2, -1, 0.25]], dtype=np.float32))
    c = o.gemm_f32acc(a, b, 0)
    assert c.tolist() == [[6.0, 0.75], [3.5, -1.5]]


@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 5, 7), (17, 33, 40), (64, 80, 129), (130, 70, 300)])
def test_layouts_agree_and_match_fp64(shape):
    M, N, K = shape
    rng = np.random.default_rng(M * 1000 + N * 10 + K)
    a = o.f32_to_bf16(rng.uniform(-1, 1, (M, K)).astype(np.float32))
    b = o.f32_to_bf16(rng.uniform(-1, 1, (N, K)).astype(np.float32))
    c_nk = o.gemm_bf16(a, b, 0)
    c_kn = o.gemm_bf16(a, np.ascontiguousarray(b.T), 1)
    assert np.array_equal(c_nk, c_kn)
    c64, sabs = o.gemm_f64(a, b, 0)
    c32 = o.gemm_f32acc(a, b, 0)
    # fp32 accumulation error is bounded by ~K * 2^-24 * sum|a*b|.
    assert np.all(np.abs(c32 - c64) <= K * 2.0 ** -24 * sabs + 1e-30)
    check_parity(c_nk, c64, c_nk, ctx=str(shape))


def test_k_zero_and_empty():
    a = np.zeros((4, 0), dtype=np.uint16)
    b = np.zeros((3, 0), dtype=np.uint16)
    assert np.array_equal(o.gemm_f32acc(a, b, 0), np.zeros((4, 3), np.float32))
    assert o.gemm_bf16(np.zeros((0, 8), np.uint16), np.zeros((5, 8), np.uint16), 0).shape == (0, 5)


def _golden_files():
    return sorted(glob.glob(os.path.join(GOLDEN, "v8_*.npz")))


def test_golden_fixtures_present():
    assert _golden_files(), "tests/golden/*.npz missing (made by tests/golden/make_golden.py on a B200)"


@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: os.path.basename(p))
def test_oracle_matches_reference_kernel_outputs(path):
    """Pin: the CPU restatement reproduces what the reference's matmul_v8_tuned
    (compiled for sm_100a from its own sources) produced on a B200."""
    z = np.load(path)
    a, b, c_ref = z["A"], z["B"], z["C_ref_v8_tuned"]
    c_or = o.gemm_bf16(a, b, 0)
    c64, _ = o.gemm_f64(a, b, 0)
    stats = check_parity(c_ref, c64, c_or, ctx=os.path.basename(path))
    # The reference and the oracle round the same fp32-accumulated value; they may
    # only disagree where summation order moves a value across a rounding boundary.
    assert stats["frac_diff"] < 0.01
    if "C_cublas" in z.files:
        check_parity(z["C_cublas"], c64, c_or, ctx=os.path.basename(path) + " cublas")
