"""Shared helpers for the tests: seeded inputs and the parity tolerances.

Tolerances (the BASELINE north_star, made precise):
  * elementwise: |C - C_true| <= 2 bf16 ulp of C_true, where C_true is the
    near-exact (fp64-accumulated) product and the ulp is taken at
    max(|C_true|, rms(C_true) * 2^-8).  The floor keeps entries that cancel
    to almost zero from demanding more than fp32 accumulation can give.
  * relative Frobenius error <= 1e-3, measured against bf16_RN(C_oracle32):
    rounding an exact result to bf16 alone costs ~1.6e-3 relative Frobenius,
    so the comparison has to be made between two bf16-rounded results.
  * against the oracle's own bf16 output: at most 1 bf16 ulp anywhere, and
    the fraction of differing elements below 1% (only rounding-boundary
    cases can differ, because summation order differs).  Two fp32
    accumulations in different orders drift apart like sqrt(K): from
    K = 16384 on, entries that cancel to near the rms * 2^-8 floor can land
    2 bf16 ulp apart, so callers pass max_ulp_vs_oracle = 2 there (the bound
    against the fp64 product is unchanged).
"""
from __future__ import annotations

import numpy as np
import torch


def uniform_bf16(shape, seed: int, lo: float = -1.0, hi: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(shape, generator=g, dtype=torch.float32) * (hi - lo) + lo).to(torch.bfloat16)


def normal_bf16(shape, seed: int, std: float = 1.0) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g, dtype=torch.float32) * std).to(torch.bfloat16)


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> contiguous numpy uint16 bit patterns (CPU copy)."""
    return t.detach().to("cpu").contiguous().view(torch.int16).numpy().view(np.uint16)


def from_bits(u: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(u).view(np.int16)).view(torch.bfloat16)


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers at |x| (8 significant bits)."""
    ax = np.abs(np.asarray(x, dtype=np.float64))
    ax = np.where(ax < 2.0 ** -126, 2.0 ** -126, ax)
    return np.exp2(np.floor(np.log2(ax)) - 7)


def bf16_bits_to_f64(u: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(u).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def check_parity(c_bits: np.ndarray, c_true: np.ndarray, c_oracle_bits: np.ndarray, ctx: str = "",
                 max_ulp_vs_oracle: float = 1.0) -> dict:
    """Assert the three parity criteria; return the measured figures."""
    c = bf16_bits_to_f64(c_bits)
    o = bf16_bits_to_f64(c_oracle_bits)
    rms = float(np.sqrt(np.mean(c_true ** 2))) if c_true.size else 0.0
    floor = rms * 2.0 ** -8
    tol = 2.0 * bf16_ulp(np.maximum(np.abs(c_true), floor))
    err = np.abs(c - c_true)
    worst = float(np.max(err / tol)) if err.size else 0.0
    assert np.all(np.isfinite(c)), f"{ctx}: non-finite output"
    assert worst <= 1.0, f"{ctx}: max |dC| = {worst:.3f} x (2 bf16 ulp) > 1"
    denom = float(np.linalg.norm(c_true)) or 1.0
    frob = float(np.linalg.norm(c - o)) / denom
    assert frob <= 1e-3, f"{ctx}: relative Frobenius vs bf16(oracle) = {frob:.3e} > 1e-3"
    d_ulp = np.abs(c - o) / bf16_ulp(np.maximum(np.abs(o), floor))
    max_ulp = float(d_ulp.max()) if d_ulp.size else 0.0
    frac = float(np.mean(c_bits != c_oracle_bits)) if c_bits.size else 0.0
    assert max_ulp <= max_ulp_vs_oracle + 1e-9, f"{ctx}: {max_ulp:.2f} bf16 ulp from the oracle"
    assert frac < 0.01, f"{ctx}: {frac:.3%} of elements differ from the oracle"
    return {"max_err_over_tol": worst, "rel_frob": frob, "max_ulp_vs_oracle": max_ulp, "frac_diff": frac}


def free_port() -> int:
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def spawn_ranks(fn, make_args, nprocs: int):
    """torch.multiprocessing.spawn of `nprocs` ranks with a fresh rendezvous
    port (make_args(port) builds the argument tuple).  A port can be taken by
    another process between choosing and binding it; that case (EADDRINUSE)
    is retried with a new port, any other failure is raised."""
    import torch.multiprocessing as mp
    for attempt in range(4):
        try:
            return mp.spawn(fn, args=make_args(free_port()), nprocs=nprocs, join=True)
        except mp.ProcessRaisedException as e:
            if "EADDRINUSE" in str(e) and attempt < 3:
                continue
            raise
