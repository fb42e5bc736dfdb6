"""GPU test of b200_gemm_bf16_noalloc, the entry point for callers that cannot
allocate device memory where they multiply (a serving engine that reserved
all of HBM at start-up and keeps cudaMalloc off its request path, or a plugin
handed buffers but no allocator).  It runs the split-K GEMM with its scratch
in a static array inside the library.

Called through the C ABI.  Each case makes two calls in a row on the same
stream and checks both against the existing entry point
(b200_gemm_bf16_ws, given its own workspace from torch), bit for bit since both
run the same split plan, and against the CPU oracle with the tolerances the
other parity tests use (tests/_util.py).
This file is collected last (tests/test_zz_*), and it does not depend on any
state left by other tests.
"""
import ctypes

import numpy as np
import pytest
import torch

import b200_gemm
from b200_gemm import _lib
from oracle import oracle as o
from tests._util import bits, check_parity, uniform_bf16

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _call(fn, a, b, c, layout, *extra):
    M, K = a.shape
    N = c.shape[1]
    s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return fn(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, a.stride(0), b.stride(0), c.stride(0),
              0 if layout == "nk" else 1, *extra, s)


# (shape, layout, whether the shape's last wave is split along K on a B200)
CASES = [((4096, 4096, 4096), "kn", True), ((4096, 4096, 4096), "nk", True), ((5000, 4096, 4096), "kn", True),
         ((1000, 520, 4104), "nk", False), ((300, 600, 200), "kn", False), ((64, 4096, 4096), "nk", False)]


@pytest.mark.parametrize("shape,layout,splits", CASES,
                         ids=lambda v: "x".join(map(str, v)) if isinstance(v, tuple) else str(v))
def test_no_alloc_matches_existing_entry_point(shape, layout, splits):
    lib = _lib.load()
    b200_gemm.set_kernel("auto")
    M, N, K = shape
    a = uniform_bf16((M, K), 101)
    b_nk = uniform_bf16((N, K), 102)
    b = b_nk if layout == "nk" else b_nk.t().contiguous()
    ad, bd = a.to(DEV), b.to(DEV)

    # Existing entry point with a caller workspace (same split-K plan).
    ws_bytes = b200_gemm.ops.workspace_bytes(M, N, K, layout)
    # The split shapes really go through the scratch: a plan exists and it fits
    # the static array (16 MiB).
    assert (ws_bytes > 0) == splits
    assert ws_bytes <= 16 << 20
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=DEV)
    ws_ptr = ctypes.c_void_p((ws.data_ptr() + 255) // 256 * 256 if ws_bytes else None)
    c_ref = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    assert _call(lib.b200_gemm_bf16_ws, ad, bd, c_ref, layout, ws_ptr, ws_bytes) == _lib.B200_OK

    outs = []
    for _ in range(2):  # two calls in a row share the static scratch
        c = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device=DEV)
        assert _call(lib.b200_gemm_bf16_noalloc, ad, bd, c, layout) == _lib.B200_OK
        outs.append(c)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0

    ref_bits = bits(c_ref)
    rows = torch.arange(M) if M <= 512 else torch.tensor(sorted({0, M - 1, *range(7, M, M // 61)}))
    c_or = o.gemm_bf16(bits(a[rows]), bits(b_nk), 0)
    c64, _ = o.gemm_f64(bits(a[rows]), bits(b_nk), 0)
    for c in outs:
        cb = bits(c)
        # against the existing entry point: bit for bit (the same split plan,
        # partials added in the same fixed order; a split plan that silently
        # fell back to sequential K would differ on split shapes)
        assert np.array_equal(cb, ref_bits), f"{np.mean(cb != ref_bits):.4%} of elements differ from b200_gemm_bf16_ws"
        # against the CPU oracle on sampled rows
        check_parity(cb[rows.numpy()], c64, c_or, ctx=f"noalloc {shape} {layout}")
