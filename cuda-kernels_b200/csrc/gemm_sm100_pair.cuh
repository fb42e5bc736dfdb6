// CTA-pair (cta_group::2) variant of the persistent BF16 GEMM for sm_100a.
//
// Same contract as gemm_sm100.cuh (C = A x op(B), bf16 in, fp32 accumulate,
// bf16 out, B either [N,K] or [K,N]), but each output tile of 256 x BN is
// computed by the two CTAs of a cluster together:
//
//   * CTA r (r = 0, 1) TMA-loads rows [128r, 128r+128) of the A tile and
//     columns [r*BN/2, (r+1)*BN/2) of the B tile into its own shared memory.
//     Both CTAs' loads signal the leader's (r = 0) "full" barrier.  Each CTA
//     therefore streams half of B instead of all of it, which halves the B
//     traffic per SM relative to a 128 x BN single-CTA tile with the same
//     accumulator size.  Loads are plain (one destination each).
//   * One thread of the leader issues tcgen05.mma.cta_group::2 with M = 256:
//     the tensor cores of both SMs read both CTAs' operand halves and each
//     SM accumulates its own 128 rows x BN columns in its own TMEM.
//   * The leader's tcgen05.commit (one instruction signalling both CTAs'
//     barriers) releases ring stages and hands finished accumulators to the
//     epilogue warps of both CTAs; each CTA's epilogue
//     drains its own TMEM and TMA-stores its 128 rows.  The accumulator is
//     double-buffered in TMEM so the epilogue overlaps the next tile.
//
// Every mbarrier wait is bounded (ptx_sm100.cuh: mbar_wait).  The only
// unbounded waits are the two full-cluster barriers at set-up and teardown,
// which every thread of both CTAs reaches because all other waits end.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "gemm_sm100.cuh"
#include "ptx_sm100.cuh"

namespace b200 {

constexpr int kPairBM = 256;  // rows of C per pair tile (128 per CTA)

// The 256 x 512 tile with eight epilogue warps (384 threads): warps 0-3 hold
// the producer and the MMA issuer and give registers away, warps 4-11 drain
// the accumulator, two per TMEM lane quarter, one per 256-column half.  Each
// epilogue thread pulls its row's 256 columns out of TMEM into 128 registers
// of packed bf16 and frees its half of the accumulator at once; the C stores
// then leave from registers while the next tile's MMAs already run (with
// four epilogue warps the next tile waited for the stores: all CTAs drain at
// the same moment and the stores are slow).  Register shares: 128 threads x
// 56 + 256 x 224 = 384 x 168, the pool of a launch at 168 registers; the
// host uses this kernel only when the binary has that count.
constexpr int kWide8Threads = 384;
constexpr uint32_t kWide8RegsLaunch = 168, kWide8RegsOther = 56, kWide8RegsEpi = 224;
static_assert(128 * kWide8RegsOther + 256 * kWide8RegsEpi <= kWide8Threads * kWide8RegsLaunch,
              "register reallocation exceeds the launch pool");

template <int BN, int STAGES>
struct PairSmemPlan {
  // A tile of BN columns is computed as kNSub pair MMAs of N = 256 each
  // (N = 256 is the UMMA maximum).  For sub-tile h, CTA r holds the B columns
  // [h*256 + r*128, h*256 + r*128 + 128) of the tile, so TMEM column c of the
  // accumulator is tile column c.
  static constexpr int kMmaN = BN < 256 ? BN : 256;
  static constexpr int kNSub = BN / kMmaN;
  static constexpr int kSubCols = kMmaN / 2;            // B columns per CTA per sub-tile
  static constexpr int kHalfN = BN / 2;                  // B columns per CTA
  // Accumulator buffers in TMEM: two (the epilogue of one tile overlaps the
  // next tile's MMAs) when they fit, else one whose sub-tiles are released
  // one by one.
  static constexpr int kAccN = 2 * BN <= kTmemCols ? 2 : 1;
  static constexpr int kABytes = kBM * kBK * 2;        // this CTA's 128 rows of A: 16 KiB
  static constexpr int kBSubBytes = kSubCols * kBK * 2;  // one sub-tile's B columns of this CTA
  static constexpr int kBBytes = kNSub * kBSubBytes;     // 16 KiB (BN = 256) or 32 KiB (BN = 512)
  static constexpr int kStageBytes = kABytes + kBBytes;  // per CTA
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + STAGES * kABytes;
  static constexpr int kOffC = kOffB + STAGES * kBBytes;
  static constexpr int kOffBar = kOffC + kEpiWarps * 2 * kEpiBufBytes;
  // barriers: full[STAGES], empty[STAGES], acc_full[kAccN], acc_empty[kAccN][kNSub], drain
  static constexpr int kNumBars = 2 * STAGES + kAccN + kAccN * kNSub + 1;
  static constexpr int kOffTmemHolder = kOffBar + kNumBars * 8;
  static constexpr int kOffAbort = kOffTmemHolder + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAllocBytes = kBytes + 1024;
  static_assert(kAllocBytes <= 232448, "shared memory plan exceeds 227 KiB");
  static_assert(kSubCols % 64 == 0, "each CTA's B columns per sub-tile must be whole 64-column swizzle atoms");
  static_assert(kAccN * BN <= kTmemCols, "accumulators must fit in TMEM");
};

// Kernel body, shared by the plain/fused kernel (one output map) and the
// gathering kernel (one output map per rank: every C tile is stored to each).
template <int BN, int STAGES, bool B_MN, bool EPI, int EW = 4>
__device__ __forceinline__ void pair_gemm_body(const CUtensorMap& tmA, const CUtensorMap& tmB,
                                               const CUtensorMap* outs, const int n_out, const GemmParams& p) {
  using Plan = PairSmemPlan<BN, STAGES>;
  constexpr int kNSub = Plan::kNSub;
  constexpr int kAccN = Plan::kAccN;
  static_assert(BN == 256 || BN == 512, "pair tiles are 256 x 256 or 256 x 512");
  static_assert(EW == 4 || (EW == 8 && BN == 512 && !EPI), "eight epilogue warps: plain 256 x 512 tiles only");

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_u32);

  const uint32_t sA = base + Plan::kOffA;
  const uint32_t sB = base + Plan::kOffB;
  const uint32_t sC = base + Plan::kOffC;
  const uint32_t bar0 = base + Plan::kOffBar;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto accf_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto acce_bar = [&](int b, int h) { return bar0 + 8u * (2 * STAGES + kAccN + b * kNSub + h); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + kAccN + kAccN * kNSub);
  volatile uint32_t* tmem_holder = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffTmemHolder);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_ctarank();  // 0 = MMA leader of the pair
  const int pair = blockIdx.x >> 1;
  const int num_pairs = gridDim.x >> 1;

  // ---- set-up -------------------------------------------------------------
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);   // leader's producer arrive + both CTAs' transaction bytes
      mbar_init(empty_bar(s), 1);  // one commit from the leader's MMA thread
    }
    for (int b = 0; b < kAccN; ++b) {
      mbar_init(accf_bar(b), 1);  // one commit from the leader's MMA thread
      for (int h = 0; h < kNSub; ++h) mbar_init(acce_bar(b, h), 2 * kEpiWarps);  // every epilogue warp of the pair
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    for (int i = 0; i < n_out; ++i) tma_prefetch_desc(outs + i);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(const_cast<uint32_t*>(tmem_holder)), kTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive / transaction
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  // Launched with programmatic stream serialisation: the prologue above ran
  // while the previous kernel in the stream may still be finishing; wait for
  // it before touching global memory, and let the next kernel start its own
  // prologue as early as possible.  (An L2 prefetch of the first operand
  // tiles before the wait measured neutral here and 6 % slower on the skinny
  // kernel; there is none.)
  pdl_launch_dependents();
  pdl_wait();

  // Warps 0-1 (with eight epilogue warps: the whole first warpgroup, 0-3,
  // which gives registers to the epilogue warpgroups) produce and issue.
  if (warp < (EW == 8 ? 4 : 2)) {
  if constexpr (EW == 8) setmaxnreg_dec<kWide8RegsOther>();
  if (warp == 0) {
    // ---- TMA producer (both CTAs) ---------------------------------------------
    if (lane == 0) {
      // Operand tiles are re-read by the other tiles of their row / column
      // block: keep them in L2 ahead of the output stream (B200: 2-3 % at
      // 4096^3 and 8192^3, from fewer DRAM trips under the power cap).
      const uint64_t pol = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      // B filled by other GPUs (exchange hooks): its flags before any load.
      if (p.n_dep > 0 && !wait_deps(p)) {
        raise_status(p, abort_flag, kDevTimeoutPeer);
        ok = false;
      }
      for (int w = pair; w < p.num_work && ok; w += num_pairs) {
        const WorkItem wk = work_item(w, p);
        const int row0 = wk.mb * kPairBM + (int)rank * kBM;
        const int col0 = wk.nb * BN + (int)rank * Plan::kSubCols;  // + h * kMmaN for sub-tile h
        for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = mapa_shared(full_bar(stage), 0);
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), 2 * Plan::kStageBytes);
          tma_load_2d_pair(sA + stage * Plan::kABytes, &tmA, fb, kb * kBK, row0, pol);
#pragma unroll
          for (int h = 0; h < kNSub; ++h) {
            const uint32_t dstB = sB + stage * Plan::kBBytes + h * Plan::kBSubBytes;
            const int colh = col0 + h * Plan::kMmaN;
            if constexpr (!B_MN) {
              tma_load_2d_pair(dstB, &tmB, fb, kb * kBK, colh, pol);
            } else {
#pragma unroll
              for (int j = 0; j < Plan::kSubCols / 64; ++j) {
                tma_load_2d_pair(dstB + j * (64 * kBK * 2), &tmB, fb, colh + 64 * j, kb * kBK, pol);
              }
            }
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) raise_status(p, abort_flag, kDevTimeoutProducer);
      // Drain (leader): the leader's full barriers count the bytes of both CTAs'
      // loads, so once the most recent phase of each has completed, nothing
      // either CTA loaded is still in flight.  The follower's own loads are
      // covered by this wait plus the teardown cluster barrier.
      if (rank == 0) {
        const uint32_t nst = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
        for (uint32_t i = 0; i < nst; ++i) {
          const uint32_t it = issued - 1u - i;
          if (!mbar_wait(full_bar(it % STAGES), (it / STAGES) & 1u, p.timeout_ns, nullptr)) {
            raise_status(p, abort_flag, kDevTimeoutDrain);
            break;
          }
        }
        // Every load of this pair has landed: B's slot is no longer read here.
        release_slot(p, num_pairs);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer (leader CTA only) ---------------------------------------------
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kPairBM, Plan::kMmaN, false, B_MN);
      // Descriptors of stage 0; later stages and K slices only move the
      // start-address field (bits 0..13, address >> 4), which never carries.
      //   A, K-major SW128: 128-byte rows, 8-row groups 1024 B apart; the k-th
      //     16-wide K slice starts 32 B into each row.
      //   B, K-major: same as A.  B, MN-major ([K,N] source): 64-column atoms
      //     8 KiB apart (LBO), 8-row K groups 1024 B apart (SBO); the k-th K
      //     slice starts 16 rows = 2 KiB on.
      const uint64_t a_desc0 = smem_desc_sw128(sA, 16, 1024);
      const uint64_t b_desc0 = B_MN ? smem_desc_sw128(sB, 64 * kBK * 2, 1024) : smem_desc_sw128(sB, 16, 1024);
      constexpr uint32_t kBStep = B_MN ? (2048 >> 4) : (32 >> 4);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int w = pair; w < p.num_work && ok; w += num_pairs) {
        const WorkItem wk = work_item(w, p);
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        // Sub-tile h of this accumulator may be written once the epilogue has
        // drained it (checked right before its first MMA of the tile).
        bool free_h[kNSub];
#pragma unroll
        for (int h = 0; h < kNSub; ++h) free_h[h] = false;
        for (int kb = wk.kb0; kb < wk.kb1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + (uint64_t)((stage * Plan::kABytes) >> 4);
          const uint64_t bd = b_desc0 + (uint64_t)((stage * Plan::kBBytes) >> 4);
#pragma unroll
          for (int h = 0; h < kNSub; ++h) {
            if (!free_h[h]) {
              if (!mbar_wait(acce_bar(acc, h), acc_phase ^ 1u, p.timeout_ns, abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              free_h[h] = true;
            }
            const uint64_t bdh = bd + (uint64_t)((h * Plan::kBSubBytes) >> 4);
#pragma unroll
            for (int k = 0; k < kBK / kUmmaK; ++k) {
              umma_bf16_pair(d_tmem + (uint32_t)(h * Plan::kMmaN), ad + 2u * k, bdh + kBStep * k, idesc,
                             (kb != wk.kb0 || k != 0) ? 1u : 0u);
            }
          }
          if (!ok) break;
          // Stage `stage` is free in both CTAs once these MMAs have read it.
          umma_commit_pair_both(empty_bar(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit_pair_both(accf_bar(acc));  // accumulator ready for both CTAs' epilogues
        if (++acc == kAccN) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) raise_status(p, abort_flag, kDevTimeoutMma);
      umma_commit_pair(mapa_shared(drain_bar, 0));
      if (!mbar_wait(drain_bar, 0u, p.timeout_ns, nullptr)) raise_status(p, abort_flag, kDevTimeoutDrain);
    }
    __syncwarp();
  }
  } else if constexpr (EW == 8) {
    // ---- epilogue, eight warps (4..11 of both CTAs): whole halves into registers ----
    setmaxnreg_inc<kWide8RegsEpi>();
    {
      const int ew = warp - 4;
      const int q = warp & 3;  // TMEM lane quarter
      const int h = ew >> 2;   // accumulator half: columns [256 h, 256 h + 256)
      const uint32_t tmem_lane = (uint32_t)(q * 32) << 16;
      const uint32_t buf = sC + (uint32_t)(ew * kEpiBufBytes);  // one 4 KiB staging buffer per warp
      uint32_t acc_phase = 0;
      for (int w = pair; w < p.num_work; w += num_pairs) {
        const WorkItem wk = work_item(w, p);
        const bool got = mbar_wait(accf_bar(0), acc_phase, p.timeout_ns, abort_flag);
        if (!named_bar_and(2, 8 * 32, got)) {
          if (lane == 0) raise_status(p, abort_flag, kDevTimeoutEpilogue);
          break;
        }
        tc_fence_after();
        const uint32_t t_row = tmem_base + tmem_lane + (uint32_t)(h * Plan::kMmaN);
        uint32_t pk[128];  // this row's 256 columns as packed bf16 pairs
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r0[32], r1[32];
          tmem_ld_32x32b_x32(t_row + c * kEpiCols, r0);
          tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, r1);
          tmem_ld_wait_regs(r0);
          tmem_ld_wait_regs(r1);
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(__uint_as_float(r0[2 * k]), __uint_as_float(r0[2 * k + 1]));
            __nv_bfloat162 hi = __floats2bfloat162_rn(__uint_as_float(r1[2 * k]), __uint_as_float(r1[2 * k + 1]));
            pk[c * 32 + k] = *reinterpret_cast<uint32_t*>(&lo);
            pk[c * 32 + 16 + k] = *reinterpret_cast<uint32_t*>(&hi);
          }
        }
        // This half of the accumulator is in registers: hand it back now.
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(acce_bar(0, h), 0));
        const int row = wk.mb * kPairBM + (int)rank * kBM + q * kEpiRowsPerWarp;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (lane == 0) bulk_wait_group_read<0>();  // the previous store has read `buf`
          __syncwarp();
          const uint32_t row_addr = buf + lane * 128u;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t dst = row_addr + (((uint32_t)j ^ (lane & 7u)) << 4);
            asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(pk[c * 32 + 4 * j]),
                         "r"(pk[c * 32 + 4 * j + 1]), "r"(pk[c * 32 + 4 * j + 2]), "r"(pk[c * 32 + 4 * j + 3])
                         : "memory");
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(outs, buf, wk.nb * BN + h * Plan::kMmaN + c * kEpiCols, row);
            bulk_commit_group();
          }
        }
        acc_phase ^= 1u;
      }
      if (lane == 0) bulk_wait_group_read<0>();  // smem reads done; the global writes complete with the grid
      __syncwarp();
    }
  } else {
    // ---- epilogue (warps 2..5 of both CTAs) ------------------------------------------
    const int q = warp & 3;
    const int slot = warp - 2;
    const uint32_t tmem_lane = (uint32_t)(q * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    int sbuf = 0;
    for (int w = pair; w < p.num_work; w += num_pairs) {
      const WorkItem wk = work_item(w, p);
      if constexpr (EPI) {
        if (wk.part < 0 || wk.part == p.sk_parts - 1) {
          epilogue_prefetch_row(p.epi, wk.mb * kPairBM + (int)rank * kBM + q * kEpiRowsPerWarp + (int)lane,
                                wk.nb * BN, BN, p.M, p.N);
        }
      }
      const bool got = mbar_wait(accf_bar(acc), acc_phase, p.timeout_ns, abort_flag);
      // All four epilogue warps take the same decision (they meet at named
      // barriers below, so none may leave the loop alone).
      if (!named_bar_and(2, kEpiWarps * 32, got)) {
        if (lane == 0) raise_status(p, abort_flag, kDevTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + tmem_lane + (uint32_t)(acc * BN);
      const int row_local = q * kEpiRowsPerWarp + (int)lane;  // row of this CTA's 128-row half
      const int row = wk.mb * kPairBM + (int)rank * kBM + q * kEpiRowsPerWarp;
      // Split-K slots of this CTA: partial of part j lives at slot (split, j, rank).
      const bool sk_writer = wk.part >= 0 && wk.part < p.sk_parts - 1;
      const bool sk_finisher = wk.part >= 0 && wk.part == p.sk_parts - 1;
      auto slot_index = [&](int j) { return (wk.split * (p.sk_parts - 1) + j) * 2 + (int)rank; };
      if (sk_finisher) {
        // Wait until every earlier part of this tile has published its partial.
        if (warp == 2 && lane == 0) {
          for (int j = 0; j < p.sk_parts - 1; ++j) {
            if (!wait_flag_eq(p.flags + slot_index(j), p.epoch, p.timeout_ns)) {
              raise_status(p, abort_flag, kDevTimeoutSplitK);
              break;
            }
          }
        }
        named_bar_sync(1, kEpiWarps * 32);
      }
#pragma unroll 1
      for (int c = 0; c < BN / kEpiCols; ++c) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, r0);
        tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, r1);
        tmem_ld_wait_regs(r0);
        tmem_ld_wait_regs(r1);
        if (((c + 1) * kEpiCols) % Plan::kMmaN == 0) {
          // Sub-tile (c * 64) / 256 of this accumulator is drained: hand it back.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(mapa_shared(acce_bar(acc, (c * kEpiCols) / Plan::kMmaN), 0));
        }
        if (sk_writer) {
          // fp32 partial, layout [BN/4][128 rows][4]: a warp's 32 rows of one
          // 4-column group are 512 contiguous bytes.
          float* dst = p.workspace + (size_t)slot_index(wk.part) * (size_t)(kBM * BN);
#pragma unroll
          for (int g = 0; g < 16; ++g) {
            const uint32_t* src = g < 8 ? &r0[g * 4] : &r1[(g - 8) * 4];
            st_global_v4(dst + ((size_t)(c * 16 + g) * kBM + row_local) * 4, __uint_as_float(src[0]),
                         __uint_as_float(src[1]), __uint_as_float(src[2]), __uint_as_float(src[3]));
          }
          continue;
        }
        if (sk_finisher) {
          // Add the earlier parts' partials in part order (deterministic).
          for (int j = 0; j < p.sk_parts - 1; ++j) {
            const float* src = p.workspace + (size_t)slot_index(j) * (size_t)(kBM * BN);
#pragma unroll
            for (int g = 0; g < 16; ++g) {
              const float4 v = ld_global_cg_v4(src + ((size_t)(c * 16 + g) * kBM + row_local) * 4);
              uint32_t* d = g < 8 ? &r0[g * 4] : &r1[(g - 8) * 4];
              d[0] = __float_as_uint(__uint_as_float(d[0]) + v.x);
              d[1] = __float_as_uint(__uint_as_float(d[1]) + v.y);
              d[2] = __float_as_uint(__uint_as_float(d[2]) + v.z);
              d[3] = __float_as_uint(__uint_as_float(d[3]) + v.w);
            }
          }
        }
        const int n0 = wk.nb * BN + c * kEpiCols;
        if constexpr (EPI) {
          if (p.epi.active) {
            epilogue_row32(r0, p.epi, row + (int)lane, n0, p.M, p.N);
            epilogue_row32(r1, p.epi, row + (int)lane, n0 + 32, p.M, p.N);
          }
        }
        const bool f32 = EPI && p.epi.out_f32 != 0;
        // bf16 D alternates the warp's two buffers; fp32 D uses both per chunk.
        const uint32_t buf0 = sC + (uint32_t)((slot * 2 + (f32 ? 0 : sbuf)) * kEpiBufBytes);
        const uint32_t buf1 = sC + (uint32_t)((slot * 2 + 1) * kEpiBufBytes);
        if (lane == 0) {
          if (f32) {
            bulk_wait_group_read<0>();
          } else {
            bulk_wait_group_read<1>();  // the store that used `buf0` has read it
          }
        }
        __syncwarp();
        stage_row64(r0, r1, f32, buf0, buf1, lane);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          for (int i = 0; i < n_out; ++i) {
            tma_store_2d(outs + i, buf0, n0, row);
            if (f32) tma_store_2d(outs + i, buf1, n0 + 32, row);
          }
          bulk_commit_group();
        }
        sbuf ^= 1;
      }
      if (sk_writer) {
        // Publish: every epilogue thread's partial stores happen-before the
        // release of the flag (barrier, then a release store at GPU scope).
        named_bar_sync(1, kEpiWarps * 32);
        if (warp == 2 && lane == 0) st_release_gpu(p.flags + slot_index(wk.part), p.epoch);
      }
      if (++acc == kAccN) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) {
      if (n_out > 1) {
        // Gathering: the stores into other GPUs' memory are complete and
        // visible system-wide before this CTA exits.
        bulk_wait_group<0>();
        __threadfence_system();
      } else {
        bulk_wait_group_read<0>();  // smem reads done; the global writes complete with the grid
      }
    }
    __syncwarp();
  }

  // ---- teardown -------------------------------------------------------------
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its barriers or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int BN, int STAGES, bool B_MN, bool EPI = false>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                          const __grid_constant__ CUtensorMap tmC, const __grid_constant__ GemmParams p) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, (uint32_t)kDevWrongArch);
#else
  pair_gemm_body<BN, STAGES, B_MN, EPI>(tmA, tmB, &tmC, 1, p);
#endif
}

// 256 x 512 tiles, plain epilogue, eight epilogue warps (see kWide8Threads).
template <bool B_MN>
__global__ void __launch_bounds__(kWide8Threads, 1)
    gemm_bf16_pair_wide8_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ GemmParams p) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, (uint32_t)kDevWrongArch);
#else
  pair_gemm_body<512, 4, B_MN, false, 8>(tmA, tmB, &tmC, 1, p);
#endif
}

// Row-sharded GEMM with the C all-gather fused in: 256 x 256 pair tiles
// (double-buffered accumulators keep the MMAs running while the epilogue
// stores each tile p.num_out times), every tile stored to each rank's
// gathered C through `outs`.
template <bool B_MN>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_bf16_pair_gather_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                                 const __grid_constant__ OutMaps outs, const __grid_constant__ GemmParams p) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, (uint32_t)kDevWrongArch);
#else
  pair_gemm_body<256, 6, B_MN, false>(tmA, tmB, outs.m, p.num_out, p);
#endif
}

}  // namespace b200
