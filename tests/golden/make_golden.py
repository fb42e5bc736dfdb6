"""Make the golden fixtures that pin the CPU oracle to the reference itself.

Run on a B200 from the repo root:  python tests/golden/make_golden.py
Needs oracle/_ref/libref_v8_tuned.so (built by `make -C oracle ref` from the
reference's own bf16_matmul/matmul_v8_tuned.cu for sm_100a).

Each fixture holds seeded bf16 inputs A [M,K] and B [N,K] (the reference's
layout), the reference kernel's output C_ref_v8_tuned = A @ B^T, and cuBLAS's
output (torch.matmul on the GPU, the check the reference's main.py uses,
bf16_matmul/main.py:31,54).  Shapes obey the reference's tile assert
(M % 128 == N % 64 == K % 64 == 0, matmul_v8_tuned.cu:238).
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as o  # noqa: E402
from tests._util import bits, normal_bf16, uniform_bf16  # noqa: E402

CASES = [
    # name, M, N, K, distribution, seed
    ("v8_128x64x64_uniform", 128, 64, 64, "uniform", 11),
    ("v8_256x128x192_normal", 256, 128, 192, "normal", 12),
    ("v8_128x192x512_uniform", 128, 192, 512, "uniform", 13),
    ("v8_384x64x256_normal", 384, 64, 256, "normal", 14),
]


def main() -> int:
    lib = o.ref_lib()
    for name, M, N, K, dist, seed in CASES:
        gen = uniform_bf16 if dist == "uniform" else normal_bf16
        a = gen((M, K), seed)
        b = gen((N, K), seed + 1000)
        ad, bd = a.cuda(), b.cuda()
        cd = torch.empty((M, N), dtype=torch.bfloat16, device="cuda")
        torch.cuda.synchronize()
        rc = lib.ref_matmul_v8_tuned(ad.data_ptr(), bd.data_ptr(), cd.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        if rc != 0:
            raise RuntimeError(f"{name}: reference kernel returned {rc}")
        cub = torch.matmul(ad, bd.t().contiguous())
        torch.cuda.synchronize()
        np.savez_compressed(os.path.join(HERE, name + ".npz"), A=bits(a), B=bits(b), C_ref_v8_tuned=bits(cd),
                            C_cublas=bits(cub), meta=np.array([M, N, K, seed]))
        print("wrote", name)
    return 0


if __name__ == "__main__":
    sys.exit(main())
