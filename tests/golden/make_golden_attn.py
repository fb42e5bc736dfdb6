"""Make the golden fixtures that pin the attention oracle to the reference itself.

Run on a B200 from the repo root:
    python tests/golden/make_golden_attn.py [OUT_DIR]      (default: tests/golden)
Needs oracle/_ref/ref_fa2.so (built by oracle/build_ref_fa2.py from the
reference's own flash_attn/flash_attn.cpp and fa2_tma_lazy_rescale.cu for
sm_100a).

Each fixture holds seeded bf16 inputs Q [batch, seq, heads, 128] and K, V
[batch, seq, kv_heads, 128], the reference operator's output
O_ref = fa2_tma_lazy_rescale(Q, K, V) (causal, flash_attn/flash_attn.cpp:16-30)
and torch SDPA's output on the same GPU (the check the reference's main.py
makes, flash_attn/main.py:36-47).
"""
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import build_ref_fa2  # noqa: E402
from tests._util import bits  # noqa: E402

CASES = [
    # name, batch, seq, heads, kv_heads, seed
    ("fa2_1x128x2_mha", 1, 128, 2, 2, 21),
    ("fa2_1x192x4_gqa2", 1, 192, 4, 2, 22),
    ("fa2_2x256x2_mha", 2, 256, 2, 2, 23),
]


def main() -> int:
    out_dir = sys.argv[1] if len(sys.argv) > 1 else HERE
    os.makedirs(out_dir, exist_ok=True)
    ref = build_ref_fa2.load()
    for name, B, S, H, Hkv, seed in CASES:
        g = torch.Generator().manual_seed(seed)
        q = torch.randn((B, S, H, 128), generator=g).to(torch.bfloat16)
        k = torch.randn((B, S, Hkv, 128), generator=g).to(torch.bfloat16)
        v = torch.randn((B, S, Hkv, 128), generator=g).to(torch.bfloat16)
        qd, kd, vd = q.cuda(), k.cuda(), v.cuda()
        o_ref = ref.fa2_tma_lazy_rescale(qd, kd, vd)
        rep = H // Hkv
        o_sdpa = F.scaled_dot_product_attention(qd.transpose(1, 2), kd.repeat_interleave(rep, 2).transpose(1, 2),
                                                vd.repeat_interleave(rep, 2).transpose(1, 2),
                                                is_causal=True).transpose(1, 2)
        torch.cuda.synchronize()
        np.savez_compressed(os.path.join(out_dir, name + ".npz"), Q=bits(q), K=bits(k), V=bits(v),
                            O_ref_fa2=bits(o_ref), O_sdpa=bits(o_sdpa))
        err = (o_ref.float() - o_sdpa.float()).abs().max().item()
        print(f"{name}: max |O_ref - O_sdpa| = {err:.4f}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
