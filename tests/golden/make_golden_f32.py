"""Make the golden fixtures that pin the fp32 CPU oracle to the reference itself.

Run on a B200 from the repo root:
    python tests/golden/make_golden_f32.py [OUT_DIR]      (default: tests/golden)
Needs oracle/_ref/libref_f32.so (built by `make -C oracle ref` from the
reference's own fp32_matmul/matmul.cu for sm_100a).

Each fixture holds seeded fp32 inputs A [M,K] and B [K,N] (row-major, the
reference's layout, fp32_matmul/matmul.cpp:20-33), the reference's v1 output
(one thread per element, an fp32 multiply-add chain over k in order,
fp32_matmul/matmul.cu:18-36), its v5 output where the shape is whole tiles,
and cuBLAS's fp32 output (torch.matmul with TF32 off, the reference's check,
fp32_matmul/main.py:22-29).
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import oracle as o  # noqa: E402

CASES = [
    # name, M, N, K, seed
    ("f32_37x53x301", 37, 53, 301, 31),
    ("f32_128x128x256", 128, 128, 256, 32),
    ("f32_256x128x96", 256, 128, 96, 33),
]


def main() -> int:
    out_dir = sys.argv[1] if len(sys.argv) > 1 else HERE
    os.makedirs(out_dir, exist_ok=True)
    lib = o.ref_f32_lib()
    torch.backends.cuda.matmul.allow_tf32 = False
    for name, M, N, K, seed in CASES:
        g = torch.Generator().manual_seed(seed)
        a = torch.randn((M, K), generator=g)
        b = torch.randn((K, N), generator=g)
        ad, bd = a.cuda(), b.cuda()
        c1 = torch.empty((M, N), device="cuda")
        c5 = torch.full((M, N), float("nan"), device="cuda")
        torch.cuda.synchronize()
        if lib.ref_matmul_f32_v1(ad.data_ptr(), bd.data_ptr(), c1.data_ptr(), M, N, K) != 0:
            raise RuntimeError(f"{name}: reference v1 failed")
        rc5 = lib.ref_matmul_f32_v5(ad.data_ptr(), bd.data_ptr(), c5.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        cub = torch.matmul(ad, bd)
        torch.cuda.synchronize()
        arrays = dict(A=a.numpy(), B=b.numpy(), C_ref_v1=c1.cpu().numpy(), C_cublas=cub.cpu().numpy())
        if rc5 == 0:
            arrays["C_ref_v5"] = c5.cpu().numpy()
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), **arrays)
        same = np.mean(arrays["C_ref_v1"] == o.gemm_f32(arrays["A"], arrays["B"], 1))
        print(f"{name}: v1 bit-equal to the oracle on {same:.2%} of elements; v5 {'stored' if rc5 == 0 else 'n/a'}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
