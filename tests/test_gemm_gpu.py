"""GPU parity tests of the B200 GEMM, called through the C ABI (b200_gemm.gemm
wraps b200_gemm_bf16 via ctypes), against:
  * the CPU oracle (oracle/gemm_oracle.c) and its fp64 product,
  * the reference's own matmul_v8_tuned rebuilt for sm_100a (oracle/_ref),
  * cuBLAS (torch.matmul), the check the reference's main.py makes
    (bf16_matmul/main.py:44-54).
Tolerances are stated in tests/_util.py (check_parity).
"""
import numpy as np
import pytest
import torch

import b200_gemm
from oracle import oracle as o
from tests._util import bits, check_parity, normal_bf16, uniform_bf16

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _pad8(x: int) -> int:
    return max((x + 7) // 8 * 8, 8)


def _padded(t: torch.Tensor) -> torch.Tensor:
    """Device copy of a 2-D bf16 tensor with its row pitch rounded up to 8 elements."""
    r, c = t.shape
    buf = torch.zeros((r, _pad8(c)), dtype=torch.bfloat16, device=DEV)
    buf[:, :c] = t.to(DEV)
    return buf[:, :c]


def _run(a, b, layout):
    """Run the GPU GEMM on padded device copies; returns the bf16 result on the CPU."""
    ad, bd = _padded(a), _padded(b)
    M = a.shape[0]
    N = b.shape[0] if layout == "nk" else b.shape[1]
    out = torch.full((M, _pad8(N)), float("nan"), dtype=torch.bfloat16, device=DEV)[:, :N]
    res = b200_gemm.gemm(ad, bd, b_layout=layout, out=out)
    assert res.data_ptr() == out.data_ptr()
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    return out.cpu()


def _make(M, N, K, layout, seed, dist="uniform"):
    gen = uniform_bf16 if dist == "uniform" else normal_bf16
    a = gen((M, K), seed)
    b_nk = gen((N, K), seed + 7)
    b = b_nk if layout == "nk" else b_nk.t().contiguous()
    return a, b, b_nk


EDGE_SHAPES = [
    (1, 1, 1), (1, 8, 8), (5, 3, 7), (8, 8, 8), (16, 24, 40), (128, 256, 64), (127, 255, 63),
    (129, 257, 65), (128, 64, 128), (200, 300, 136), (256, 512, 192), (300, 600, 200),
    (1000, 72, 40), (64, 100, 1000), (131, 517, 333),
]


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("shape", EDGE_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_edge_shapes_vs_oracle(shape, layout):
    M, N, K = shape
    a, b, b_nk = _make(M, N, K, layout, seed=M * 7919 + N * 31 + K)
    c = _run(a, b, layout)
    c_or = o.gemm_bf16(bits(a), bits(b_nk), 0)
    c64, _ = o.gemm_f64(bits(a), bits(b_nk), 0)
    check_parity(bits(c), c64, c_or, ctx=f"{shape} {layout}")


def _sampled_parity(a, b_nk, c, rows, ctx):
    a_s = bits(a[rows])
    c_or = o.gemm_bf16(a_s, bits(b_nk), 0)
    c64, _ = o.gemm_f64(a_s, bits(b_nk), 0)
    return check_parity(bits(c[rows]), c64, c_or, ctx=ctx)


def _rows(M, n, seed):
    rng = np.random.default_rng(seed)
    r = set(rng.choice(M, size=min(n, M), replace=False).tolist()) | {0, M - 1}
    return torch.tensor(sorted(r))


@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("shape", [(2048, 4096, 128), (4096, 4096, 64), (1024, 1024, 8192), (640, 2560, 520),
                                   (4100, 4000, 200), (4096, 4136, 72)],
                         ids=lambda s: "x".join(map(str, s)))
def test_persistent_multi_tile_vs_oracle(shape, layout):
    """More tiles than SMs (each CTA loops over several tiles, both TMEM
    accumulator buffers and every ring stage wrap), checked on sampled rows."""
    M, N, K = shape
    a, b, b_nk = _make(M, N, K, layout, seed=K + N)
    c = _run(a, b, layout)
    _sampled_parity(a, b_nk, c, _rows(M, 48, M + K), ctx=f"{shape} {layout}")


@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_headline_4096_full_oracle(layout):
    """M=N=K=4096, U(-1,1) bf16, every element against the oracle."""
    M = N = K = 4096
    a, b, b_nk = _make(M, N, K, layout, seed=4096)
    c = _run(a, b, layout)
    c_or = o.gemm_bf16(bits(a), bits(b_nk), 0)
    c32 = o.gemm_f32acc(bits(a), bits(b_nk), 0).astype(np.float64)
    check_parity(bits(c), c32, c_or, ctx=f"4096^3 {layout}")


@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (256, 128, 192), (1024, 2048, 512), (8192, 4096, 1024)],
                         ids=lambda s: "x".join(map(str, s)))
def test_vs_reference_kernel(shape):
    """Same seeded inputs through the reference's matmul_v8_tuned (sm_100a rebuild)."""
    if not o.ref_available():
        pytest.skip("oracle/_ref/libref_v8_tuned.so not built")
    M, N, K = shape
    a = normal_bf16((M, K), 5).to(DEV)
    b = normal_bf16((N, K), 6).to(DEV)
    c_ref = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    torch.cuda.synchronize()
    assert o.ref_lib().ref_matmul_v8_tuned(a.data_ptr(), b.data_ptr(), c_ref.data_ptr(), M, N, K) == 0
    torch.cuda.synchronize()
    c = b200_gemm.matmul(a, b)
    torch.cuda.synchronize()
    cb, rb = bits(c), bits(c_ref)
    x = (cb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    y = (rb.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    from tests._util import bf16_ulp
    d = np.abs(x - y) / bf16_ulp(np.maximum(np.abs(y), np.sqrt(np.mean(y ** 2)) * 2 ** -8))
    assert d.max() <= 1.0, f"max {d.max():.2f} ulp from matmul_v8_tuned"
    assert np.mean(cb != rb) < 0.01


def test_vs_cublas_like_reference_main():
    """The reference's own correctness gate: assert_close against torch.matmul
    with default bf16 tolerances on N(0,1) 4096x4096 inputs (bf16_matmul/main.py:27-54)."""
    a = torch.randn((4096, 4096), dtype=torch.bfloat16, generator=torch.Generator().manual_seed(1)).to(DEV)
    b = torch.randn((4096, 4096), dtype=torch.bfloat16, generator=torch.Generator().manual_seed(2)).to(DEV)
    ref = torch.matmul(a, b.transpose(0, 1).contiguous())
    out = b200_gemm.matmul(a, b)
    torch.testing.assert_close(out, ref)
    out_kn = b200_gemm.gemm(a, b.transpose(0, 1).contiguous(), b_layout="kn")
    torch.testing.assert_close(out_kn, ref)


def test_torch_binding_matches_c_abi():
    from b200_gemm.binding import load_binding
    ext = load_binding()
    a = uniform_bf16((300, 520), 1).to(DEV)
    b = uniform_bf16((200, 520), 2).to(DEV)
    c1 = ext.matmul_b200(a, b)
    c2 = b200_gemm.matmul(a, b)
    c3 = ext.matmul_b200_kn(a, b.t().contiguous())
    torch.cuda.synchronize()
    assert c1.shape == (300, 200)  # N from B.size(0), unlike the reference's B.size(1)
    assert torch.equal(c1, c2) and torch.equal(c1, c3)
    with pytest.raises(ValueError, match="bfloat16"):
        ext.matmul_b200(a.float(), b)
    with pytest.raises(ValueError, match="inner dimensions differ"):
        ext.matmul_b200(a, b[:, :100])
    with pytest.raises(ValueError, match="CUDA"):
        ext.matmul_b200(a.cpu(), b.cpu())


def test_k_zero_m_zero_and_streams():
    a = torch.empty((64, 0), dtype=torch.bfloat16, device=DEV)
    b = torch.empty((32, 0), dtype=torch.bfloat16, device=DEV)
    c = torch.full((64, 32), 3.0, dtype=torch.bfloat16, device=DEV)
    b200_gemm.gemm(a, b, out=c)
    torch.cuda.synchronize()
    assert torch.count_nonzero(c) == 0
    e = b200_gemm.gemm(torch.empty((0, 16), dtype=torch.bfloat16, device=DEV),
                       torch.ones((8, 16), dtype=torch.bfloat16, device=DEV))
    assert e.shape == (0, 8)
    # a side stream: result must be ready after synchronising that stream only
    s = torch.cuda.Stream()
    a = uniform_bf16((512, 256), 3).to(DEV)
    b = uniform_bf16((384, 256), 4).to(DEV)
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        c = b200_gemm.matmul(a, b)
    s.synchronize()
    ref = o.gemm_bf16(bits(a.cpu()), bits(b.cpu()), 0)
    assert np.mean(bits(c) != ref) < 0.01


def test_strided_views_and_errors():
    base = uniform_bf16((256, 640), 9).to(DEV)
    a = base[:, 64:64 + 320]  # lda = 640, offset 128 bytes
    b = uniform_bf16((96, 320), 10).to(DEV)
    out_buf = torch.zeros((256, 200), dtype=torch.bfloat16, device=DEV)
    out = out_buf[:, 8:8 + 96]
    b200_gemm.gemm(a, b, out=out)
    torch.cuda.synchronize()
    ref = o.gemm_bf16(bits(a.cpu()), bits(b.cpu()), 0)
    assert np.mean(bits(out) != ref) < 0.01
    assert torch.count_nonzero(out_buf[:, :8]) == 0 and torch.count_nonzero(out_buf[:, 104:]) == 0
    with pytest.raises(b200_gemm.B200GemmError):
        b200_gemm.gemm(base[:, 1:321], b)  # 2-byte offset: not 16-byte aligned
    with pytest.raises(ValueError):
        b200_gemm.gemm(a, b.t())  # not row-major


@pytest.fixture
def forced_kernel():
    """Yields a setter for the kernel override and restores automatic selection afterwards."""
    yield b200_gemm.set_kernel
    b200_gemm.set_kernel("auto")


FORCE_SHAPES = [(1, 8, 8), (5, 3, 7), (17, 129, 70), (100, 300, 136), (128, 256, 1000), (129, 257, 65),
                (300, 520, 200)]


@pytest.mark.parametrize("kernel", ["single", "pair", "skinny"])
@pytest.mark.parametrize("layout", ["nk", "kn"])
@pytest.mark.parametrize("shape", FORCE_SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_every_kernel_path_vs_oracle(shape, layout, kernel, forced_kernel):
    """Each of the three kernels computes the same product on ragged shapes."""
    M, N, K = shape
    if kernel == "skinny" and M > 128:
        forced_kernel("skinny")
        a = torch.zeros((M, 8), dtype=torch.bfloat16, device=DEV)
        with pytest.raises(b200_gemm.B200GemmError):
            b200_gemm.matmul(a, torch.zeros((8, 8), dtype=torch.bfloat16, device=DEV))
        return
    forced_kernel(kernel)
    a, b, b_nk = _make(M, N, K, layout, seed=M + 3 * N + 7 * K)
    c = _run(a, b, layout)
    c_or = o.gemm_bf16(bits(a), bits(b_nk), 0)
    c64, _ = o.gemm_f64(bits(a), bits(b_nk), 0)
    check_parity(bits(c), c64, c_or, ctx=f"{shape} {layout} {kernel}")


SKINNY_CFG = [(m, n, k) for m in (16, 64, 128) for (n, k) in ((4096, 4096), (14336, 4096), (4096, 14336))]


@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("shape", SKINNY_CFG, ids=lambda s: "x".join(map(str, s)))
def test_baseline_skinny_configs_vs_oracle(shape, layout):
    """A ~ N(0,1), B ~ N(0, 1/K), every element against the oracle."""
    M, N, K = shape
    a = normal_bf16((M, K), M + N)
    b_nk = normal_bf16((N, K), K + 1, std=K ** -0.5)
    b = b_nk if layout == "nk" else b_nk.t().contiguous()
    c = b200_gemm.gemm(a.to(DEV), b.to(DEV), b_layout=layout)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    c_or = o.gemm_bf16(bits(a), bits(b_nk), 0)
    c32 = o.gemm_f32acc(bits(a), bits(b_nk), 0).astype(np.float64)
    check_parity(bits(c), c32, c_or, ctx=f"{shape} {layout}")


@pytest.mark.parametrize("M", [1, 3, 16, 31, 48, 65, 127, 128])
def test_skinny_split_k_vs_oracle(M):
    """Small M with K long enough for a multi-CTA cluster split and a ragged last split."""
    N, K = 1000, 3000
    a = uniform_bf16((M, K), M)
    b = uniform_bf16((N, K), M + 1)
    c = _run(a, b, "nk")
    c_or = o.gemm_bf16(bits(a), bits(b), 0)
    c64, _ = o.gemm_f64(bits(a), bits(b), 0)
    check_parity(bits(c), c64, c_or, ctx=f"M={M}")


def test_device_wait_timeout_is_reported_and_context_survives():
    """A bounded device wait on a barrier nothing arrives at gives up after its
    limit; the host reads B200_ERR_DEVICE_TIMEOUT and the GPU keeps working."""
    import ctypes
    import time
    from b200_gemm import _lib
    lib = _lib.load()
    assert b200_gemm.check_status() == 0
    s = torch.cuda.current_stream()
    t0 = time.time()
    assert lib.b200_gemm_selftest_wait_timeout(200_000_000, ctypes.c_void_p(s.cuda_stream)) == 0  # 0.2 s
    bits_ = ctypes.c_uint32(0)
    rc = lib.b200_gemm_status(ctypes.c_void_p(s.cuda_stream), ctypes.byref(bits_))
    dt = time.time() - t0
    assert rc == _lib.B200_ERR_DEVICE_TIMEOUT and bits_.value != 0
    assert 0.15 < dt < 5.0, dt
    assert b200_gemm.check_status() == 0  # the status word was cleared by the read
    a = uniform_bf16((256, 128), 1).to(DEV)
    b = uniform_bf16((64, 128), 2).to(DEV)
    c = b200_gemm.matmul(a, b)
    torch.cuda.synchronize()
    assert np.mean(bits(c) != o.gemm_bf16(bits(a.cpu()), bits(b.cpu()), 0)) < 0.01


def _raw_gemm(a, b, c, layout, ws=None, ws_bytes=0):
    import ctypes
    from b200_gemm import _lib
    lib = _lib.load()
    M, K = a.shape
    N = c.shape[1]
    s = torch.cuda.current_stream().cuda_stream
    if ws is None:
        return lib.b200_gemm_bf16(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, a.stride(0), b.stride(0),
                                  c.stride(0), 0 if layout == "nk" else 1, ctypes.c_void_p(s))
    return lib.b200_gemm_bf16_ws(a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, a.stride(0), b.stride(0),
                                 c.stride(0), 0 if layout == "nk" else 1, ctypes.c_void_p(ws), ws_bytes,
                                 ctypes.c_void_p(s))


@pytest.mark.parametrize("shape", [(4096, 4096, 4096), (1024, 1024, 8192), (640, 2560, 2056), (300, 520, 4100),
                                   (129, 257, 2060), (5000, 4096, 4096)], ids=lambda s: "x".join(map(str, s)))
@pytest.mark.parametrize("layout", ["nk", "kn"])
def test_split_k_tail_matches_oracle_and_is_deterministic(shape, layout, forced_kernel):
    """The last wave's tiles split along K across pairs (b200_gemm_bf16_ws):
    same product as without the split (both against the oracle), and two
    calls give identical bits (partials are added in a fixed order).  The
    pair kernel is forced: small shapes would otherwise take 128 x 64 tiles,
    which have no split-K tail."""
    forced_kernel("pair")
    M, N, K = shape
    ws_bytes = b200_gemm.ops.workspace_bytes(M, N, K, layout)
    assert ws_bytes > 0, "shape chosen to exercise the split-K tail"
    a, b, b_nk = _make(M, N, K, layout, seed=M + N + K)
    ad, bd = _padded(a), _padded(b)  # row pitches rounded up to 8 elements
    ws = torch.empty(max(ws_bytes, 1) + 256, dtype=torch.uint8, device=DEV)
    ws_ptr = (ws.data_ptr() + 255) // 256 * 256

    def out():
        return torch.zeros((M, _pad8(N)), dtype=torch.bfloat16, device=DEV)[:, :N]
    c_split, c_split2, c_plain = out(), out(), out()
    assert _raw_gemm(ad, bd, c_split, layout, ws_ptr, ws_bytes) == 0
    ws.fill_(0xAB)  # leftover bytes in the workspace must not matter
    assert _raw_gemm(ad, bd, c_split2, layout, ws_ptr, ws_bytes) == 0
    assert _raw_gemm(ad, bd, c_plain, layout) == 0
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    assert torch.equal(c_split, c_split2)
    rows = _rows(M, 64, K) if M > 512 else torch.arange(M)
    for c, ctx in ((c_split, "split"), (c_plain, "plain")):
        _sampled_parity(a, b_nk, c.cpu(), rows, ctx=f"{shape} {layout} {ctx}")


def test_split_k_workspace_arguments():
    from b200_gemm import _lib
    M = N = K = 4096
    ws_bytes = b200_gemm.ops.workspace_bytes(M, N, K, "nk")
    assert 0 < ws_bytes < 32 << 20
    a = uniform_bf16((M, K), 1).to(DEV)
    b = uniform_bf16((N, K), 2).to(DEV)
    ws = torch.empty(ws_bytes + 512, dtype=torch.uint8, device=DEV)
    base = (ws.data_ptr() + 255) // 256 * 256
    c_small = torch.empty((M, N), dtype=torch.bfloat16, device=DEV)
    c_ref = torch.empty_like(c_small)
    assert _raw_gemm(a, b, c_small, "nk", base, ws_bytes - 1) == 0   # too small: runs without the split
    assert _raw_gemm(a, b, c_ref, "nk") == 0
    assert _raw_gemm(a, b, c_ref, "nk", base + 16, ws_bytes) == _lib.B200_ERR_ALIGNMENT
    torch.cuda.synchronize()
    assert torch.equal(c_small, c_ref)
    assert b200_gemm.ops.workspace_bytes(64, 4096, 4096, "nk") == 0  # skinny kernel: no split-K tail


# BASELINE configs 2, 4 and 5 at their real sizes, where the dispatcher picks
# other tiles than at 4096^3: 8192^3 and 16384^3 (square sweep), the
# projection shapes with the widest N (128256: a ragged last 512-column tile,
# over 2000 column blocks) and the ragged M = 8191 / 5000 on the 256 x 512
# path, and the one-GPU panel of the row-sharded job (16384 x 8192 x 8192).
# Inputs are generated on the GPU (seeded); every column of sampled rows
# (first, last and random ones) is checked against the oracle with the bounds
# of tests/_util.check_parity.
LARGE_CONFIGS = [
    (8192, 8192, 8192, "uniform"), (16384, 16384, 16384, "uniform"), (16384, 8192, 8192, "uniform"),
    (8192, 128256, 4096, "normal"), (8191, 28672, 4096, "normal"), (8191, 4096, 14336, "normal"),
    (5000, 128256, 4096, "normal"), (8191, 6144, 4096, "normal"),
]


def _dev_inputs(M, N, K, layout, dist, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    b_shape = (K, N) if layout == "kn" else (N, K)
    if dist == "uniform":
        a = (torch.rand((M, K), generator=g, device=DEV) * 2 - 1).to(torch.bfloat16)
        b = (torch.rand(b_shape, generator=g, device=DEV) * 2 - 1).to(torch.bfloat16)
    else:  # activations N(0, 1), weights N(0, 1/K)
        a = torch.randn((M, K), generator=g, device=DEV).to(torch.bfloat16)
        b = (torch.randn(b_shape, generator=g, device=DEV) * K ** -0.5).to(torch.bfloat16)
    return a, b


@pytest.mark.parametrize("layout", ["kn", "nk"])
@pytest.mark.parametrize("cfg", LARGE_CONFIGS, ids=lambda c: "x".join(map(str, c[:3])))
def test_baseline_large_configs_sampled_rows(cfg, layout):
    M, N, K, dist = cfg
    a, b = _dev_inputs(M, N, K, layout, dist, seed=M + N + K)
    c = b200_gemm.gemm(a, b, b_layout=layout)
    torch.cuda.synchronize()
    assert b200_gemm.check_status() == 0
    rows = _rows(M, 24, M * 3 + K).to(DEV)
    a_s = bits(a[rows])
    b_bits = bits(b)
    lay = 1 if layout == "kn" else 0
    c_or = o.gemm_bf16(a_s, b_bits, lay)
    c64, _ = o.gemm_f64(a_s, b_bits, lay)
    check_parity(bits(c[rows]), c64, c_or, ctx=f"{M}x{N}x{K} {layout}",
                 max_ulp_vs_oracle=2.0 if K >= 16384 else 1.0)
    del a, b, c
    torch.cuda.empty_cache()

