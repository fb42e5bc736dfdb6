"""GPU parity tests of the flash attention forward (b200_flash_attn_bf16, the
reference's flash_attn operator): against the exact fp64 attention of the same
bf16 inputs (oracle.attention) with the reference's own tolerance
(assert_close rtol = atol = 1e-2, flash_attn/main.py:46) plus a mean-error
bound, and against torch's scaled_dot_product_attention on a large case.
Covers causal and full masks, ragged sequence lengths (tiles of 128), several
batches and heads, and scores that grow along the keys so the lazy rescaling
of the running max is exercised."""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import b200_gemm
from oracle import oracle as o
from tests._util import bits

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _inputs(B, S, H, seed, grow=False):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, S, H, 128), generator=g)
    k = torch.randn((B, S, H, 128), generator=g)
    v = torch.randn((B, S, H, 128), generator=g)
    if grow:  # later keys score higher: the row max keeps rising, forcing rescales
        k = k * torch.linspace(0.5, 6.0, S).view(1, S, 1, 1)
    return q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("shape", [(1, 128, 2), (2, 384, 3), (1, 200, 2), (1, 1024, 4), (1, 77, 1)],
                         ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("grow", [False, True])
def test_attention_vs_exact(shape, causal, grow):
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
