"""GPU parity tests of the flash attention forward (b200_flash_attn_bf16, the
reference's flash_attn operator): against the exact fp64 attention of the same
bf16 inputs (oracle.attention) with the reference's own tolerance
(assert_close rtol = atol = 1e-2, flash_attn/main.py:46) plus a mean-error
bound, and against torch's scaled_dot_product_attention on a large case.
Covers causal and full masks, ragged sequence lengths (tiles of 128), several
batches and heads, grouped-query attention (fewer key/value heads than query
heads, as the reference's kernel allows), the reference-shaped torch binding
(fa2_tma_lazy_rescale), and scores that grow along the keys so the lazy
rescaling of the running max is exercised.  The exact-oracle cases run on
both kernels (one CTA per two query tiles, and CTA pairs per four), forced
through flash_attn_set_kernel; the automatic choice is covered by the rest."""
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import b200_gemm
from oracle import oracle as o
from tests._util import bits, from_bits

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(params=["single", "pair"])
def attn_kernel(request):
    b200_gemm.flash_attn_set_kernel(request.param)
    yield request.param
    b200_gemm.flash_attn_set_kernel("auto")


def _inputs(B, S, H, seed, grow=False, Hkv=None):
    Hkv = H if Hkv is None else Hkv
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, S, H, 128), generator=g)
    k = torch.randn((B, S, Hkv, 128), generator=g)
    v = torch.randn((B, S, Hkv, 128), generator=g)
    if grow:  # later keys score higher: the row max keeps rising, forcing rescales
        k = k * torch.linspace(0.5, 6.0, S).view(1, S, 1, 1)
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("shape", [(1, 128, 2), (2, 384, 3), (1, 200, 2), (1, 1024, 4), (1, 77, 1), (1, 1, 2),
                                   (3, 130, 5), (1, 640, 2), (1, 2178, 2)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("grow", [False, True])
def test_attention_vs_exact(shape, causal, grow, attn_kernel):
    B, S, H = shape
    q, k, v = _inputs(B, S, H, seed=B * 1000 + S + H, grow=grow)
    out = b200_gemm.flash_attn(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    exact = o.attention(bits(q), bits(k), bits(v), causal)
    got = out.float().cpu().numpy().astype(np.float64)
    assert np.all(np.isfinite(got))
    err = np.abs(got - exact)
    assert np.all(err <= 1e-2 + 1e-2 * np.abs(exact)), f"max err {err.max():.4f}"
    assert err.mean() < 2e-3, f"mean err {err.mean():.5f}"


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("shape", [(1, 256, 4, 2), (2, 200, 6, 1), (1, 384, 8, 4), (1, 1100, 4, 2)],
                         ids=lambda s: "x".join(map(str, s)))
def test_grouped_query_attention_vs_exact(shape, causal, attn_kernel):
    B, S, H, Hkv = shape
    q, k, v = _inputs(B, S, H, seed=17 * S + H + Hkv, Hkv=Hkv)
    out = b200_gemm.flash_attn(q.to(DEV), k.to(DEV), v.to(DEV), causal=causal)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    exact = o.attention(bits(q), bits(k), bits(v), causal)
    err = np.abs(out.float().cpu().numpy().astype(np.float64) - exact)
    assert np.all(err <= 1e-2 + 1e-2 * np.abs(exact)), f"max err {err.max():.4f}"
    assert err.mean() < 2e-3, f"mean err {err.mean():.5f}"
    # Same bits as running each query head against its repeated key/value head.
    rep = H // Hkv
    mha = b200_gemm.flash_attn(q.to(DEV), k.repeat_interleave(rep, 2).to(DEV), v.repeat_interleave(rep, 2).to(DEV),
                               causal=causal)
    assert torch.equal(out, mha)


def test_reference_binding_matches_c_abi():
    """fa2_tma_lazy_rescale(Q, K, V) of the torch binding (the reference operator's
    name and signature, flash_attn/flash_attn.cpp:16-30): causal, O allocated like Q,
    torch's current stream; bit-identical to the C-ABI call, and like the
    reference's main.py it is checked against SDPA with rtol = atol = 1e-2."""
    from b200_gemm.binding import load_attn_binding
    ext = load_attn_binding()
    q, k, v = (t.to(DEV) for t in _inputs(1, 1024, 8, seed=11))
    o_ext = ext.fa2_tma_lazy_rescale(q, k, v)
    o_abi = b200_gemm.flash_attn(q, k, v, causal=True)
    o_full = ext.flash_attn_b200(q, k, v, causal=False)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    assert o_ext.shape == q.shape and o_ext.dtype == torch.bfloat16
    assert torch.equal(o_ext, o_abi)
    assert torch.equal(o_full, b200_gemm.flash_attn(q, k, v, causal=False))
    ref = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                         is_causal=True).transpose(1, 2)
    torch.testing.assert_close(o_ext, ref, rtol=1e-2, atol=1e-2)
    # Strided (non-packed) views are packed by the binding, as the reference's
    # strided tensor maps accept them.
    qt = q.transpose(1, 2).contiguous().transpose(1, 2)
    assert torch.equal(ext.fa2_tma_lazy_rescale(qt, k, v), o_ext)


GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", ["fa2_1x128x2_mha", "fa2_1x192x4_gqa2", "fa2_2x256x2_mha"])
def test_attention_vs_reference_golden(name):
    """Against the reference operator's own outputs (fa2_tma_lazy_rescale run on a
    B200, tests/golden/make_golden_attn.py): within the reference's check, and no
    less accurate than the reference against the exact result."""
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    q, k, v = (from_bits(d[x]).to(DEV) for x in ("Q", "K", "V"))
    out = b200_gemm.flash_attn(q, k, v, causal=True)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    got = out.float().cpu().numpy().astype(np.float64)
    ref = o.bf16_to_f32(d["O_ref_fa2"]).astype(np.float64)
    assert np.all(np.abs(got - ref) <= 1e-2 + 1e-2 * np.abs(ref)), f"{name}: max {np.abs(got - ref).max():.4f}"
    exact = o.attention(d["Q"], d["K"], d["V"], True)
    ours, theirs = np.abs(got - exact).mean(), np.abs(ref - exact).mean()
    assert ours <= 1.5 * theirs + 1e-4, f"{name}: mean error {ours:.2e} vs the reference's {theirs:.2e}"


def test_attention_vs_reference_live():
    """Against the reference operator run live (oracle/_ref/ref_fa2.so, built from
    its own sources for sm_100a) on the benchmark's head layout with grouped heads."""
    path = os.path.join(os.path.dirname(GOLDEN), "..", "oracle", "_ref", "ref_fa2.so")
    if not os.path.exists(path):
        pytest.skip("oracle/_ref/ref_fa2.so not built (needs the reference sources)")
    from oracle import build_ref_fa2
    ref_mod = build_ref_fa2.load()
    q, k, v = (t.to(DEV) for t in _inputs(1, 1024, 8, seed=31, Hkv=2))
    ours = b200_gemm.flash_attn(q, k, v, causal=True)
    ref = ref_mod.fa2_tma_lazy_rescale(q, k, v)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    torch.testing.assert_close(ours, ref, rtol=1e-2, atol=1e-2)
    exact = o.attention(bits(q), bits(k), bits(v), True)
    e_ours = np.abs(ours.float().cpu().numpy() - exact).mean()
    e_ref = np.abs(ref.float().cpu().numpy() - exact).mean()
    assert e_ours <= 1.5 * e_ref + 1e-4, f"mean error {e_ours:.2e} vs the reference's {e_ref:.2e}"


def test_attention_large_vs_sdpa():
    """The reference's own benchmark shape (batch 1, 32 heads, causal) at 4096."""
    q, k, v = (t.to(DEV) for t in _inputs(1, 4096, 32, seed=7))
    out = b200_gemm.flash_attn(q, k, v, causal=True)
    ref = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                         is_causal=True).transpose(1, 2)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    torch.testing.assert_close(out, ref, rtol=1e-2, atol=1e-2)


def test_attention_argument_errors():
    q = torch.zeros((1, 128, 1, 64), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(b200_gemm.B200GemmError):
        b200_gemm.flash_attn(q, q, q)  # head_dim must be 128
    with pytest.raises(ValueError):
        b200_gemm.flash_attn(q.float(), q, q)
    q = torch.zeros((1, 128, 6, 128), dtype=torch.bfloat16, device=DEV)
    kv = torch.zeros((1, 128, 4, 128), dtype=torch.bfloat16, device=DEV)
    with pytest.raises(ValueError):
        b200_gemm.flash_attn(q, kv, kv)  # 6 query heads over 4 key/value heads
    with pytest.raises(ValueError):
        b200_gemm.flash_attn(q, kv, kv[:, :64])  # K and V differ
