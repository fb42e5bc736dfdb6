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
//     S x (N / 128) CTAs stream B concurrently.  The fp32 partial tiles are
//     reduced through distributed shared memory — no global scratch: CTA r
//     owns tile rows [r*R, (r+1)*R), R = 128 / S, and every other CTA sends it
//     their partials of those rows as one bulk shared-to-shared copy.
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
constexpr int kMaxSplits = 8;   // cluster size limit (portable)

struct SkinnyParams {
  int32_t M, N, K;
  int32_t num_k_blk;     // total K-blocks of 64
  int32_t kb_per_split;  // K-blocks per CTA of a cluster
  int32_t splits;        // S = cluster size along x: 1, 2, 4 or 8
  uint64_t timeout_ns;
  uint32_t* status;
  EpilogueParams epi;  // fused epilogue (element [m, n] of D; see gemm_sm100.cuh)
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
  static constexpr int kNumBars = 2 * STAGES + 3;  // full, empty, acc_full, drain, reduction
  static constexpr int kOffTmemHolder = kOffBar + kNumBars * 8;
  static constexpr int kOffAbort = kOffTmemHolder + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAllocBytes = kBytes + 1024;
  static constexpr int kTmemCols = MPAD <= 32 ? 32 : (MPAD <= 64 ? 64 : (MPAD <= 128 ? 128 : 256));
  // Epilogue scratch inside the (then idle) ring.  S > 1, R = 128 / S rows
  // owned per CTA, rows padded to kPitch floats (a lane moves its row with
  // 16-byte accesses; the odd number of 16-byte units per row spreads
  // consecutive rows over all banks):
  //   [0, recv)          the owned rows' partials, one block per split
  //                      ([S][R][kPitch] fp32; this CTA's own block is
  //                      staged locally, the others arrive by bulk copy);
  //   [recv, cstage)     this CTA's partials of the rows the others own
  //                      ([S-1][R][kPitch] fp32), one bulk copy per owner;
  //   [cstage, ...)      the D block of the owned rows, [MPAD][R] (bf16
  //                      or fp32).
  // S == 1: four per-warp D tiles [MPAD][32] at the start of the ring.
  static constexpr int kPitch = MPAD + 4;
  __host__ __device__ static constexpr int block_bytes(int S) { return (kSkinnyBN / S) * kPitch * 4; }
  __host__ __device__ static constexpr int recv_bytes(int S) { return S * block_bytes(S); }
  __host__ __device__ static constexpr int cstage_off(int S) {
    return S > 1 ? (recv_bytes(S) + (S - 1) * block_bytes(S) + 1023) & ~1023 : 0;
  }
  __host__ __device__ static constexpr int cstage_bytes(int S) {
    return S > 1 ? MPAD * (kSkinnyBN / S) * 4 : 4 * MPAD * 32 * 4;  // room for fp32 D
  }
  // Fused-epilogue variant only: the tile's block of C_in, [MPAD][128] bf16,
  // in its own region after the barriers, loaded while the K loop runs.
  static constexpr int kCinTileBytes = MPAD * kSkinnyBN * 2;
  static constexpr int kOffCinTile = (kBytes + 127) & ~127;
  static constexpr int kAllocBytesEpi = kOffCinTile + kCinTileBytes + 1024;
  static_assert(kAllocBytesEpi <= 232448, "fused-epilogue shared memory plan exceeds 227 KiB");
  __host__ __device__ static constexpr bool fits(int S) { return cstage_off(S) + cstage_bytes(S) <= kRingBytes; }
  // Largest power-of-two split count (<= 8) whose reduction scratch fits.
  __host__ __device__ static constexpr int max_splits() { return fits(8) ? 8 : fits(4) ? 4 : fits(2) ? 2 : 1; }
  static_assert(kAllocBytes <= 232448, "shared memory plan exceeds 227 KiB");
  static_assert(MPAD % 16 == 0 && MPAD >= 16 && MPAD <= 256, "UMMA N must be 16..256 in steps of 16");
};

// Fused epilogue for element [m, n] of D given its C_in value (0 when not
// read): same operations and order as epilogue_row32.
__device__ __forceinline__ float skinny_epi(float x, const EpilogueParams& e, float bias_n, float cin) {
  x = __fmul_rn(e.alpha, x);
  x = __fadd_rn(x, bias_n);
  return __fadd_rn(x, __fmul_rn(e.beta, cin));
}

// Writes D element (one fp32 value) into a staging tile as bf16 or fp32.
__device__ __forceinline__ void skinny_stage(uint32_t addr_elem0, int idx, float x, bool f32) {
  if (f32) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr_elem0 + (uint32_t)(idx * 4)), "f"(x) : "memory");
  } else {
    const __nv_bfloat16 hv = __float2bfloat16_rn(x);
    const uint16_t hb = *reinterpret_cast<const uint16_t*>(&hv);
    asm volatile("st.shared.b16 [%0], %1;" ::"r"(addr_elem0 + (uint32_t)(idx * 2)), "h"(hb) : "memory");
  }
}

__device__ __forceinline__ void skinny_raise(const SkinnyParams& p, volatile uint32_t* abort_flag, uint32_t code) {
  *abort_flag = 1u;
  if (p.status != nullptr) atomicOr(p.status, code);
}

// Grid: (S, ceil(N/128)); cluster (S, 1, 1).  CTA rank r of cluster y handles
// N rows [128y, 128y+128) and K-blocks [r*kb_per_split, (r+1)*kb_per_split).
template <int MPAD, int STAGES, bool B_MN, bool EPI = false>
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
  const uint32_t red_bar = drain_bar + 8u;  // partials from the other CTAs have landed
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
    mbar_init(red_bar, 1);
    // Every other CTA of the cluster sends this CTA one block of partials.
    if (p.splits > 1) mbar_arrive_expect_tx(red_bar, (uint32_t)((p.splits - 1) * Plan::block_bytes(p.splits)));
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
  constexpr int kChunk = MPAD >= 32 ? 32 : 16;  // TMEM columns per load + wait
  const bool epi = warp >= 2;
  const int q = warp & 3;
  const int slot = warp - 2;
  const uint32_t tmem_row = tmem_base + ((uint32_t)(q * 32) << 16);
  const int row = q * 32 + (int)lane;  // this lane's tile row (TMEM lane)
  // my_kb == 0 (more splits than K-blocks): this CTA's accumulator was never
  // written; it contributes zero.
  const bool acc_valid = my_kb > 0;
  // TMEM -> registers, kChunk columns starting at column c; issue only (the
  // registers are valid after tmem_chunk_wait).  All four rows of a warp's
  // TMEM lanes move at once (sync.aligned: the whole warp executes these).
  auto tmem_chunk_issue = [&](int c, uint32_t (&v)[kChunk]) {
    if constexpr (kChunk == 32) {
      tmem_ld_32x32b_x32(tmem_row + (uint32_t)c, v);
    } else {
      tmem_ld_32x32b_x16(tmem_row + (uint32_t)c, v);
    }
  };
  auto tmem_chunk_wait = [&](uint32_t (&v)[kChunk]) {
    tmem_ld_wait_regs(v);
    if (!acc_valid) {
#pragma unroll
      for (int j = 0; j < kChunk; ++j) v[j] = 0u;
    }
  };
  // Runs body(c, v) over the MPAD columns in kChunk pieces, loading the next
  // piece from TMEM while the body consumes the current one.
  auto for_each_chunk = [&](auto&& body) {
    constexpr int kN = MPAD / kChunk;
    uint32_t v[2][kChunk];
    tmem_chunk_issue(0, v[0]);
    tmem_chunk_wait(v[0]);
#pragma unroll
    for (int i = 0; i < kN; ++i) {
      if (i + 1 < kN) tmem_chunk_issue((i + 1) * kChunk, v[(i + 1) & 1]);
      body(i * kChunk, v[i & 1]);
      if (i + 1 < kN) tmem_chunk_wait(v[(i + 1) & 1]);
    }
  };
  const int S = p.splits;
  const int R = kSkinnyBN / S;
  // Fused epilogue: while the K loop runs, the epilogue warps copy the C_in
  // block this CTA will read (every row m < M; the whole tile's 128 columns,
  // or with a split the R owned ones) into its shared-memory region,
  // [MPAD][128] bf16, with 16-byte loads.
  const uint32_t cin_tile = base + (uint32_t)Plan::kOffCinTile;
  const bool use_c = EPI && p.epi.active && p.epi.beta != 0.0f;
  if constexpr (EPI) {
    if (epi && use_c) {
      const int c_lo = S == 1 ? 0 : (int)rank * R;  // first tile column read
      const int groups = (S == 1 ? kSkinnyBN : R) / 8;
      for (int i = (int)threadIdx.x - 64; i < MPAD * groups; i += kEpiWarps * 32) {
        const int m = i / groups, col = c_lo + (i - m * groups) * 8;
        const int nn = n0 + col;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (m < p.M) {
          const __nv_bfloat16* src = p.epi.c_in + (size_t)m * (size_t)p.epi.ldc_in + nn;
          if (nn + 8 <= p.N) {
            w = ld_global_v4_u32(src);
          } else {
            uint32_t h[8];
#pragma unroll
            for (int e2 = 0; e2 < 8; ++e2) h[e2] = nn + e2 < p.N ? ld_global_u16(src + e2) : 0u;
            w = make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
          }
        }
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(cin_tile + (uint32_t)((m * kSkinnyBN + col) * 2)),
                     "r"(w.x), "r"(w.y), "r"(w.z), "r"(w.w)
                     : "memory");
      }
      named_bar_sync(1, kEpiWarps * 32);  // the block is in before any warp reads it
    }
  }
  // C_in[m, n0 + col] from the staged block.
  auto cin_at = [&](int m, int col) -> float {
    uint16_t hb;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(hb) : "r"(cin_tile + (uint32_t)((m * kSkinnyBN + col) * 2)));
    return bf16_bits_to_f32(hb);
  };
  bool have_acc = false;
  if (epi) {
    const bool got = mbar_wait(accf_bar, 0u, p.timeout_ns, abort_flag);
    have_acc = __all_sync(0xffffffffu, got);
    if (!have_acc && lane == 0) skinny_raise(p, abort_flag, kDevTimeoutEpilogue);
    tc_fence_after();
  }

  if (S == 1) {
    // Whole tile here: each warp rounds its 32 rows and stores them as one
    // [MPAD x 32] block of C.
    if (epi && have_acc) {
      const bool f32 = EPI && p.epi.out_f32 != 0;
      const uint32_t stage_buf = base + (uint32_t)(slot * MPAD * 32 * (f32 ? 4 : 2));
      const int n = n0 + row;  // weight row = column n of D
      float bias_n = 0.0f;
      if (EPI && p.epi.active && p.epi.bias != nullptr && n < p.N) {
        bias_n = bf16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(p.epi.bias) + n));
      }
      for_each_chunk([&](int c, const uint32_t (&v)[kChunk]) {
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          float x = __uint_as_float(v[j]);
          if constexpr (EPI) {
            if (p.epi.active) {
              x = skinny_epi(x, p.epi, bias_n, use_c ? cin_at(c + j, row) : 0.0f);
            }
          }
          skinny_stage(stage_buf, (c + j) * 32 + (int)lane, x, f32);
        }
      });
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d(&tmC, stage_buf, n0 + q * 32, 0);  // box {32, MPAD}; rows m >= M, columns >= N clipped
        bulk_commit_group();
        bulk_wait_group_read<0>();  // smem read done; the global writes complete with the grid
      }
      __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem_base, Plan::kTmemCols);
    }
    return;
  }

  // Split-K reduction, S = 2, 4 or 8.  Two split cluster barriers:
  //   #1 every CTA's ring is idle (all its MMAs done), so partials may be
  //      copied into it.  Each CTA arrives as soon as its own MMAs are done
  //      and stages its partials locally before waiting.
  //   #2 every copy into every CTA has landed, so no CTA leaves while its
  //      shared memory is still a copy's source or destination.  Each CTA
  //      arrives once its incoming blocks are in and rounds, stores its rows
  //      before waiting.
  const uint32_t blk = (uint32_t)Plan::block_bytes(S);
  const uint32_t recv_base = base;                                   // [S][R][kPitch]
  const uint32_t send_base = base + (uint32_t)Plan::recv_bytes(S);   // [S-1][R][kPitch]
  const uint32_t cstage = base + (uint32_t)Plan::cstage_off(S);      // bf16 [MPAD][R]
  cluster_arrive();  // #1: producer and MMA warps are past their drains here
  bool staged = false;
  if (epi) {
    if (have_acc) {
      const int owner = row / R;
      const int r_in = row - owner * R;
      const uint32_t dst_blk = owner == (int)rank ? recv_base + (uint32_t)rank * blk
                                                  : send_base + (uint32_t)(owner < (int)rank ? owner : owner - 1) * blk;
      const uint32_t dst_row = dst_blk + (uint32_t)(r_in * Plan::kPitch * 4);
      for_each_chunk([&](int c, const uint32_t (&v)[kChunk]) {
#pragma unroll
        for (int j = 0; j < kChunk; j += 4) {
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst_row + (uint32_t)((c + j) * 4)),
                       "r"(v[j]), "r"(v[j + 1]), "r"(v[j + 2]), "r"(v[j + 3])
                       : "memory");
        }
      });
    }
    fence_proxy_async_smem();  // staged partials -> visible to the bulk copies
    tc_fence_before();         // TMEM reads of this CTA are done before teardown
    staged = named_bar_and(1, kEpiWarps * 32, have_acc);
  }
  cluster_wait();  // #1
  if (epi && staged && warp == 2 && (int)lane < S - 1) {
    const int o = (int)lane < (int)rank ? (int)lane : (int)lane + 1;  // owner this lane sends to
    bulk_copy_to_cluster(mapa_shared(recv_base + (uint32_t)rank * blk, (uint32_t)o), send_base + lane * blk, blk,
                         mapa_shared(red_bar, (uint32_t)o));
  }
  // Owner phase mapping: the 128 epilogue threads split the owned block,
  // thread t takes row t % R and CPT consecutive columns.  With a fused
  // epilogue its bias and C_in values are loaded now, while the partials
  // are still arriving.
  constexpr int kMinCpt = 4;
  constexpr int kMaxCpt = MPAD / 2 > kMinCpt ? MPAD / 2 : kMinCpt;  // R <= 64
  const int cpt = max(kMinCpt, MPAD * R / (kEpiWarps * 32));
  const int t = (int)threadIdx.x - 64;
  const bool owner_thread = epi && t >= 0 && t < R * (MPAD / cpt);
  const int r = owner_thread ? t % R : 0;
  const int c0 = owner_thread ? (t / R) * cpt : 0;
  const int n = n0 + (int)rank * R + r;  // column n of D
  float bias_n = 0.0f;
  if constexpr (EPI) {
    if (owner_thread && p.epi.active && p.epi.bias != nullptr && n < p.N) {
      bias_n = bf16_bits_to_f32(__ldg(reinterpret_cast<const unsigned short*>(p.epi.bias) + n));
    }
  }
  bool go = false;
  if (epi) {
    bool in = false;
    if (staged) {
      in = mbar_wait(red_bar, 0u, p.timeout_ns, abort_flag);
      if (!in) skinny_raise(p, abort_flag, kDevTimeoutEpilogue);
    }
    go = named_bar_and(2, kEpiWarps * 32, in);
  }
  if (warp == 2 && lane == 0 && !go) {
    // Error path: still let every incoming block land before this CTA can leave.
    if (!mbar_wait(red_bar, 0u, p.timeout_ns, nullptr)) skinny_raise(p, abort_flag, kDevTimeoutDrain);
  }
  cluster_arrive();  // #2
  if (epi && go) {
    // Sum the S partials of the owned rows in split order (deterministic),
    // apply the epilogue, stage D[m, n0 + rank*R + r] as [MPAD][R].
    const bool f32 = EPI && p.epi.out_f32 != 0;
    if (owner_thread) {
#pragma unroll
      for (int cc = 0; cc < kMaxCpt; cc += 4) {
        if (cc < cpt) {
          const int c = c0 + cc;
          // All S loads first (independent), then the sum in split order.
          float4 x[kMaxSplits];
#pragma unroll
          for (int sp = 0; sp < kMaxSplits; ++sp) {
            if (sp < S) {
              asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                           : "=f"(x[sp].x), "=f"(x[sp].y), "=f"(x[sp].z), "=f"(x[sp].w)
                           : "r"(recv_base + (uint32_t)sp * blk + (uint32_t)((r * Plan::kPitch + c) * 4)));
            }
          }
          float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int sp = 0; sp < kMaxSplits; ++sp) {
            if (sp < S) {
              a[0] += x[sp].x;
              a[1] += x[sp].y;
              a[2] += x[sp].z;
              a[3] += x[sp].w;
            }
          }
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            float v = a[jj];
            if constexpr (EPI) {
              if (p.epi.active) v = skinny_epi(v, p.epi, bias_n, use_c ? cin_at(c + jj, (int)rank * R + r) : 0.0f);
            }
            skinny_stage(cstage, (c + jj) * R + r, v, f32);
          }
        }
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1, kEpiWarps * 32);
    if (warp == 2 && lane == 0) {
      tma_store_2d(&tmC, cstage, n0 + (int)rank * R, 0);  // box {R, MPAD}; rows m >= M, columns >= N clipped
      bulk_commit_group();
      bulk_wait_group_read<0>();  // smem read done; the global writes complete with the grid
    }
  }
  cluster_wait();  // #2
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Plan::kTmemCols);
  }
#endif  // B200_NO_SM100A_FEATURES
}

}  // namespace b200
