// Skinny-M BF16 GEMM for sm_100a: M <= 128 rows of activations against a
// large weight matrix.  These shapes are HBM-bound (B dominates the bytes), so
// the design goal is to keep many SMs streaming B at full bandwidth.
//
//   * Swap-AB: the kernel computes C^T = B x A^T.  N (the weight rows) fills
//     the 128-row UMMA M dimension; the small M becomes the UMMA N dimension
//     (MPAD = M rounded up to 16).  B is the UMMA "A" operand (K-major for the
//     reference's [N,K] layout, MN-major for [K,N]); A is the UMMA "B"
//     operand (always K-major).
//   * Split-K inside a thread-block cluster: the S CTAs of a cluster share one
//     128-row tile of N and each takes a contiguous range of K-blocks, so
//     S x (N / 128) CTAs stream B concurrently.  Partial fp32 tiles are summed
//     in the leader CTA through distributed shared memory — no global scratch.
//   * Each CTA: warp 0 TMA producer (deep ring of plain loads), warp 1 TMEM
//     allocation + single-thread tcgen05.mma issue, warps 2..5 epilogue
//     (TMEM -> registers -> [cluster reduction] -> bf16 -> smem -> TMA store of
//     C^T tile rows, i.e. C[m, n0 .. n0+127]).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "gemm_sm100.cuh"
#include "ptx_sm100.cuh"

namespace b200 {

constexpr int kSkinnyBN = 128;  // N rows per tile (UMMA M)

struct SkinnyParams {
  int32_t M, N, K;
  int32_t num_k_blk;     // total K-blocks of 64
  int32_t kb_per_split;  // K-blocks per CTA of a cluster
  int32_t splits;        // S = cluster size along x: 1, 2, 4 or 8
  uint64_t timeout_ns;
  uint32_t* status;
};

template <int MPAD, int STAGES>
struct SkinnySmemPlan {
  static constexpr int kBtBytes = kSkinnyBN * kBK * 2;  // 16 KiB: 128 weight rows x 64 K
  static constexpr int kAtBytes = MPAD * kBK * 2;       // activation rows x 64 K
  static constexpr int kStageBytes = kBtBytes + kAtBytes;
  static constexpr int kOffBt = 0;
  static constexpr int kOffAt = STAGES * kBtBytes;
  static constexpr int kRingBytes = STAGES * kStageBytes;
  static constexpr int kOffBar = kRingBytes;
  static constexpr int kNumBars = 2 * STAGES + 2;  // full, empty, acc_full, drain
  static constexpr int kOffTmemHolder = kOffBar + kNumBars * 8;
  static constexpr int kOffAbort = kOffTmemHolder + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAllocBytes = kBytes + 1024;
  static constexpr int kTmemCols = MPAD <= 32 ? 32 : (MPAD <= 64 ? 64 : (MPAD <= 128 ? 128 : 256));
  // Epilogue scratch inside the (then idle) ring, for S splits: partials of
  // the S-1 other CTAs for this CTA's 128/S rows ([S-1][MPAD][128/S] fp32),
  // then four per-warp bf16 staging tiles ([MPAD][32] each).
  static constexpr int kStagingBytes = MPAD * 32 * 2;
  static constexpr bool fits(int S) {
    return (S - 1) * MPAD * (kSkinnyBN / S) * 4 + 4 * kStagingBytes <= kRingBytes;
  }
  // Largest power-of-two split count (<= 8) whose reduction scratch fits.
  static constexpr int max_splits() { return fits(8) ? 8 : fits(4) ? 4 : fits(2) ? 2 : 1; }
  static_assert(kAllocBytes <= 232448, "shared memory plan exceeds 227 KiB");
  static_assert(MPAD % 16 == 0 && MPAD >= 16 && MPAD <= 256, "UMMA N must be 16..256 in steps of 16");
};

__device__ __forceinline__ void skinny_raise(const SkinnyParams& p, volatile uint32_t* abort_flag, uint32_t code) {
  *abort_flag = 1u;
  if (p.status != nullptr) atomicOr(p.status, code);
}

// Grid: (S, ceil(N/128)); cluster (S, 1, 1).  CTA rank r of cluster y handles
// N rows [128y, 128y+128) and K-blocks [r*kb_per_split, (r+1)*kb_per_split).
template <int MPAD, int STAGES, bool B_MN>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_bf16_skinny_kernel(const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmA,
                            const __grid_constant__ CUtensorMap tmC, const SkinnyParams p) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, (uint32_t)kDevWrongArch);
#else
  using Plan = SkinnySmemPlan<MPAD, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_u32);

  const uint32_t sBt = base + Plan::kOffBt;
  const uint32_t sAt = base + Plan::kOffAt;
  const uint32_t bar0 = base + Plan::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t accf_bar = bar0 + 8u * (2 * STAGES);
  const uint32_t drain_bar = accf_bar + 8u;
  volatile uint32_t* tmem_holder = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffTmemHolder);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_ctarank();  // split index
  const int n0 = blockIdx.y * kSkinnyBN;
  const int kb_begin = (int)rank * p.kb_per_split;
  const int kb_end = min(kb_begin + p.kb_per_split, p.num_k_blk);
  const int my_kb = max(kb_end - kb_begin, 0);

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    mbar_init(accf_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_holder)), Plan::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // Launched with programmatic stream serialisation: the prologue above ran
  // while the previous kernel in the stream may still be finishing; wait for
  // it before touching global memory, and let the next kernel start its own
  // prologue as early as possible.
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ---- TMA producer ----------------------------------------------------------
    if (lane == 0) {
      // Weights are read once: evict them first.  The activation tile is read
      // by the CTAs of every tile: keep it.
      const uint64_t pol_b = l2_policy_evict_first();
      const uint64_t pol_a = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int kb = kb_begin; kb < kb_end; ++kb) {
        if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t fb = full_bar(stage);
        mbar_arrive_expect_tx(fb, Plan::kStageBytes);
        const uint32_t dBt = sBt + stage * Plan::kBtBytes;
        if constexpr (!B_MN) {
          tma_load_2d(dBt, &tmB, fb, kb * kBK, n0, pol_b);
        } else {
          tma_load_2d(dBt, &tmB, fb, n0, kb * kBK, pol_b);
          tma_load_2d(dBt + 64 * kBK * 2, &tmB, fb, n0 + 64, kb * kBK, pol_b);
        }
        tma_load_2d(sAt + stage * Plan::kAtBytes, &tmA, fb, kb * kBK, 0, pol_a);
        ++issued;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) skinny_raise(p, abort_flag, kDevTimeoutProducer);
      const uint32_t nst = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
      for (uint32_t i = 0; i < nst; ++i) {
        const uint32_t it = issued - 1u - i;
        if (!mbar_wait(full_bar(it % STAGES), (it / STAGES) & 1u, p.timeout_ns, nullptr)) {
          skinny_raise(p, abort_flag, kDevTimeoutDrain);
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer ------------------------------------------------------------
    if (lane == 0) {
      // UMMA A = weight tile (128 x K), B = activation tile (MPAD x K), D = C^T tile.
      constexpr uint32_t idesc = idesc_bf16_f32(kSkinnyBN, MPAD, B_MN, false);
      const uint64_t a_desc0 = B_MN ? smem_desc_sw128(sBt, 64 * kBK * 2, 1024) : smem_desc_sw128(sBt, 16, 1024);
      const uint64_t b_desc0 = smem_desc_sw128(sAt, 16, 1024);
      constexpr uint32_t kAStep = B_MN ? (2048 >> 4) : (32 >> 4);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int i = 0; i < my_kb; ++i) {
        if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = a_desc0 + (uint64_t)((stage * Plan::kBtBytes) >> 4);
        const uint64_t bd = b_desc0 + (uint64_t)((stage * Plan::kAtBytes) >> 4);
#pragma unroll
        for (int k = 0; k < kBK / kUmmaK; ++k) {
          umma_bf16(tmem_base, ad + kAStep * k, bd + 2u * k, idesc, (i | k) != 0 ? 1u : 0u);
        }
        umma_commit(empty_bar(stage));
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) skinny_raise(p, abort_flag, kDevTimeoutMma);
      umma_commit(accf_bar);  // also signals when my_kb == 0 (nothing to wait for)
      umma_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0u, p.timeout_ns, nullptr)) skinny_raise(p, abort_flag, kDevTimeoutDrain);
    }
    __syncwarp();
  }

  // ---- epilogue ---------------------------------------------------------------
  // Warps 2..5 read TMEM lanes q*32 .. q*32+31, i.e. N rows n0 + q*32 + lane,
  // all MPAD columns (= rows m of C).
  const bool epi = warp >= 2;
  const int q = warp & 3;
  const int slot = warp - 2;
  const uint32_t tmem_row = tmem_base + ((uint32_t)(q * 32) << 16);
  bool have_acc = false;
  if (epi) {
    const bool got = mbar_wait(accf_bar, 0u, p.timeout_ns, abort_flag);
    have_acc = __all_sync(0xffffffffu, got);
    if (!have_acc && lane == 0) skinny_raise(p, abort_flag, kDevTimeoutEpilogue);
    tc_fence_after();
  }
  // my_kb == 0 (more splits than K-blocks): this CTA's accumulator was never
  // written; it contributes zero.
  const bool acc_valid = my_kb > 0;

  // Split-K reduction, distributed: with S = p.splits (1, 2, 4 or 8) CTA r of
  // the cluster owns tile rows [r*R, (r+1)*R), R = 128 / S, and receives the
  // other CTAs' partial sums of exactly those rows into its (then idle) ring
  // over distributed shared memory.  Two cluster barriers: the first
  // guarantees every ring is no longer read by its MMAs, the second that all
  // partials have landed.  Every CTA then rounds and stores its own rows.
  const int S = p.splits;
  const int R = kSkinnyBN / S;
  const int row = q * 32 + (int)lane;  // this lane's tile row (TMEM lane)
  const int owner = row / R;
  const int row_in_owner = row - owner * R;
  const uint32_t recv_base = base;     // [S-1 senders][MPAD][R] fp32
  auto recv_addr = [&](int sender, int owner_rank, int c, int r) {
    const int slot_ = sender < owner_rank ? sender : sender - 1;
    return recv_base + (uint32_t)(((slot_ * MPAD + c) * R + r) * 4);
  };
  auto tmem_load16 = [&](int c, uint32_t (&v)[16]) {
    if (acc_valid) {
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
          : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
            "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
          : "r"(tmem_row + (uint32_t)c));
      asm volatile(
          "tcgen05.wait::ld.sync.aligned;"
          : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]), "+r"(v[6]), "+r"(v[7]),
            "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]), "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
          :
          : "memory");
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = 0u;
    }
  };

  if (S > 1) {
    cluster_sync_all();
    if (epi && have_acc) {
      const bool remote = owner != (int)rank;
      const uint32_t dst_base = remote ? mapa_shared(recv_addr((int)rank, owner, 0, row_in_owner), (uint32_t)owner) : 0u;
#pragma unroll 1
      for (int c = 0; c < MPAD; c += 16) {
        uint32_t v[16];
        tmem_load16(c, v);  // whole warp (sync.aligned); only rows owned elsewhere are sent
        if (remote) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            asm volatile("st.shared::cluster.b32 [%0], %1;" ::"r"(dst_base + (uint32_t)((c + j) * R * 4)), "r"(v[j])
                         : "memory");
          }
        }
      }
    }
    cluster_sync_all();
  }

  // Warps holding rows this CTA owns: add the partials in split order
  // 0, 1, ..., S-1 (this CTA's own sum at position `rank`), round to bf16,
  // stage [MPAD rows m][W columns n] and TMA-store C[m, n0 + first .. +W).
  const int w_first = max(q * 32, (int)rank * R);            // first owned tile row in this warp
  const int w_end = min(q * 32 + 32, ((int)rank + 1) * R);   // one past the last
  if (epi && have_acc && w_first < w_end) {
    const int W = w_end - w_first;  // 16 or 32 columns of C
    const bool mine = row >= w_first && row < w_end;
    const uint32_t stage_buf =
        base + (uint32_t)((S - 1) * MPAD * R * 4) + (uint32_t)(slot * MPAD * 32 * 2);
#pragma unroll 1
    for (int c = 0; c < MPAD; c += 16) {
      uint32_t v[16];
      tmem_load16(c, v);
      if (mine) {
        float f[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) f[j] = 0.0f;
        for (int sp = 0; sp < S; ++sp) {
          if (sp == (int)rank) {
#pragma unroll
            for (int j = 0; j < 16; ++j) f[j] += __uint_as_float(v[j]);
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              float x;
              asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x) : "r"(recv_addr(sp, (int)rank, c + j, row_in_owner)));
              f[j] += x;
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const __nv_bfloat16 h = __float2bfloat16_rn(f[j]);
          const uint16_t hb = *reinterpret_cast<const uint16_t*>(&h);
          asm volatile("st.shared.b16 [%0], %1;" ::"r"(stage_buf + (uint32_t)(((c + j) * W + (row - w_first)) * 2)),
                       "h"(hb)
                       : "memory");
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(&tmC, stage_buf, n0 + w_first, 0);  // box {W, MPAD}; rows m >= M are clipped by TMA
      bulk_commit_group();
      bulk_wait_group_read<0>();  // smem read done; the global writes complete with the grid
    }
    __syncwarp();
  }

  tc_fence_before();
  if (p.splits > 1) {
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Plan::kTmemCols);
  }
#endif  // B200_NO_SM100A_FEATURES
}

}  // namespace b200
