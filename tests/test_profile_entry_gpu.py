"""The reference's profiling entry runs unchanged on the B200 GEMM.

oracle/Makefile builds oracle/_ref/profile_matmul_b200 from the reference's own,
unmodified bf16_matmul/profile_entry.cpp (:90-96: `profile_kernel(
PROFILE_MATMUL_SYMBOL, config)` with M = N = K = 4096, 10 warm-up launches and
one profiled launch, each followed by cudaDeviceSynchronize) and this repo's
MatmulFn launcher cuda-kernels_b200/bf16_matmul/matmul_b200.cu, with the
symbol chosen as scripts/profile.sh:95-123 chooses it (the file's basename).
Run here without a profiler: the binary must exit 0, and the launcher must
report neither a launch error nor a device-side wait that gave up (it prints
`matmul_b200: ...` on stderr for either).
"""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(REPO, "oracle", "_ref", "profile_matmul_b200")


def test_reference_profile_entry_runs_unchanged():
    if not os.path.exists(EXE):
        pytest.skip("oracle/_ref/profile_matmul_b200 not built (needs the reference's profile_entry.cpp)")
    r = subprocess.run([EXE], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, f"exit {r.returncode}: {r.stderr[-2000:]}"
    assert "matmul_b200:" not in r.stderr, r.stderr[-2000:]
    assert "error" not in r.stderr.lower(), r.stderr[-2000:]
