// FP32 GEMM on the bf16 tensor cores: each fp32 operand is split exactly into
// three bf16 parts, x = x1 + x2 + x3 (x1 and x2 the next 8 significant bits
// each, truncated; x3 the remaining 8 bits), and
//
//   A B = A3 B1 + A2 B2 + A1 B3 + A2 B1 + A1 B2 + A1 B1  (+ terms below 2^-24 |A||B|)
//
// is one bf16 GEMM with K' = 6K over concatenated operands
//   A' = [A3 | A2 | A1 | A2 | A1 | A1]   (segments along K)
//   B' = [B1 ; B2 ; B3 ; B1 ; B2 ; B1]
// accumulated in fp32 by the tensor cores and stored as fp32.  Every product
// of two bf16 parts is exact in fp32; the omitted products A2 B3, A3 B2, A3 B3
// are below fp32 rounding of the result.  The small terms come first in K so
// they are summed before the large ones.
//
// This replaces the reference's SIMT fp32 kernels (fp32_matmul/matmul.cu:18-325)
// with the B200's bf16 tensor-core path: 6x the MMA work of a bf16 GEMM, about
// 6x fewer FLOP/s than bf16 but several times the B200's fp32 SIMT rate.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

namespace b200 {

// Parts of x: 1 = top 8 significant bits, 2 = next 8, 3 = the rest (exact for
// finite normal fp32).  Inf / NaN: part 1 carries it, the others are zero.
__device__ __forceinline__ void split3_bf16(float x, uint16_t (&h)[4]) {
  const uint32_t u = __float_as_uint(x);
  h[0] = 0;
  if ((u & 0x7f800000u) == 0x7f800000u) {
    h[1] = (u & 0x007fffffu) != 0u ? (uint16_t)(0x7fc0u | ((u >> 16) & 0x8000u)) : (uint16_t)(u >> 16);
    h[2] = h[3] = 0;
    return;
  }
  h[1] = (uint16_t)(u >> 16);                              // truncate: x1
  const float r1 = x - __uint_as_float((uint32_t)h[1] << 16);  // exact
  const uint32_t v = __float_as_uint(r1);
  h[2] = (uint16_t)(v >> 16);                              // truncate: x2
  const float r2 = r1 - __uint_as_float((uint32_t)h[2] << 16);  // exact
  const __nv_bfloat16 b3 = __float2bfloat16_rn(r2);        // x3 (exact when x is normal)
  h[3] = *reinterpret_cast<const uint16_t*>(&b3);
}

// dst[r * ld_dst + c + s * seg_off] = part order[s] of src[r * ld_src + c],
// s = 0..5, for r < rows, c < cols.  `order` packs the six part numbers
// (1..3), two bits each, segment 0 in the low bits.  seg_off = K places the
// segments side by side along a row ([M,K] A, [N,K] B); seg_off = K * ld_dst
// stacks them as row blocks ([K,N] B).
__global__ void __launch_bounds__(256) split_f32_bf16x3_kernel(const float* __restrict__ src, int64_t rows,
                                                               int64_t cols, int64_t ld_src,
                                                               uint16_t* __restrict__ dst, int64_t ld_dst,
                                                               int64_t seg_off, uint32_t order) {
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const float* srow = src + r * ld_src;
    uint16_t* drow = dst + r * ld_dst;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += (int64_t)gridDim.x * blockDim.x) {
      uint16_t h[4];
      split3_bf16(srow[c], h);
#pragma unroll
      for (int s = 0; s < 6; ++s) drow[c + s * seg_off] = h[(order >> (2 * s)) & 3u];
    }
  }
}

constexpr uint32_t kSplitOrder(int p0, int p1, int p2, int p3, int p4, int p5) {
  return (uint32_t)p0 | ((uint32_t)p1 << 2) | ((uint32_t)p2 << 4) | ((uint32_t)p3 << 6) | ((uint32_t)p4 << 8) |
         ((uint32_t)p5 << 10);
}
constexpr uint32_t kSplitOrderA = kSplitOrder(3, 2, 1, 2, 1, 1);
constexpr uint32_t kSplitOrderB = kSplitOrder(1, 2, 3, 1, 2, 1);

}  // namespace b200
