// Flash attention forward on CTA pairs (tcgen05 cta_group::2): the same
// operator and arithmetic as flash_attn_fwd_kernel (attn_sm100.cuh), with
// every product issued once for two SMs.
//
// A cluster of two CTAs takes four 128-row query tiles of one (head, batch);
// CTA r holds tiles 4c + r (slot 0) and 4c + 2 + r (slot 1) and runs the
// softmax of its own rows exactly as the one-CTA kernel does.  The leader's
// MMA thread issues, per slot i and key tile j,
//   S_i  = Q_i K_j^T   M = 256 (slot i of both CTAs), N = 128 keys: each CTA
//                      holds 64 keys of K_j (its B half) and its own Q_i;
//   O_i += P_i V_j     M = 256, N = 128 head columns, A = P_i from each CTA's
//                      TMEM, each CTA holding 64 of V_j's head columns.
// So each SM reads half of every K and V tile from L2 and from its shared
// memory (a 128x128x16 share of a product reads 6 KiB of shared memory
// instead of 8 for S and 2 instead of 4 for P V).  The one-CTA kernel's
// products run at ~96 (S) and ~76 (P V) cycles per 128x128x16 step against
// 64, and this halves their operand traffic per SM; measured on B200, it does
// not make them faster: the products alone (softmax skipped, a timing copy)
// reach the same ~1300 TFLOP/s in both forms, and with the softmax the pair
// form is 25 % slower (the leader waits for the slower CTA's P every key
// tile).  So b200_flash_attn_bf16 runs this kernel only when asked
// (B200_ATTN_KERNEL_PAIR); the tests check it against the exact attention.
//
// The two tiles of a slot differ by one query tile; both run the longer
// tile's key range (for the shorter one the extra diagonal tile is fully
// masked and adds nothing to its sums).  Loads complete on the leader's
// barriers (both CTAs' bytes), commits go to both CTAs, and each CTA's
// softmax warps arrive on the leader's P barriers.  Every wait is bounded.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "attn_sm100.cuh"

namespace b200 {

constexpr int kAttnPairStages = 3;  // K and V ring depth (16 KiB halves per stage)

struct AttnPairSmemPlan {
  static constexpr int kTileBytes = 128 * 128 * 2;  // a 128 x 128 bf16 tile: 32 KiB (Q)
  static constexpr int kHalfBytes = 64 * 128 * 2;   // this CTA's half of a K or V tile: 16 KiB
  static constexpr int kOffQ = 0;                   // two Q tiles; O staging at the end
  static constexpr int kOffK = kOffQ + kAttnQTiles * kTileBytes;
  static constexpr int kOffV = kOffK + kAttnPairStages * kHalfBytes;
  static constexpr int kOffBar = kOffV + kAttnPairStages * kHalfBytes;
  // q_full[Q], k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[Q], p_full[Q][2], o_full[Q], drain
  static constexpr int kRingBars = kAttnQTiles + 4 * kAttnPairStages;
  static constexpr int kNumBars = kRingBars + 4 * kAttnQTiles + 1;
  static constexpr int kOffTmemHolder = kOffBar + kNumBars * 8;
  static constexpr int kOffAbort = kOffTmemHolder + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAllocBytes = kBytes + 1024;
  static_assert(kAllocBytes <= 232448, "pair attention shared memory plan exceeds 227 KiB");
};

// Grid (2 * heads * batch, ceil(num_q_tiles / 4)), clusters of (2, 1, 1):
// blockIdx.x / 2 is the (head, batch), blockIdx.x % 2 the CTA's rank, and
// blockIdx.y the group of four query tiles, taken in reverse order: blocks
// start x fastest, so the longest causal rows of every head start first.
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attn_fwd_pair_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                               const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                               const __grid_constant__ AttnParams p) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, (uint32_t)kDevWrongArch);
#else
  using Plan = AttnPairSmemPlan;
  constexpr int KS = kAttnPairStages;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_u32);
  const uint32_t sQ = base + Plan::kOffQ;
  const uint32_t sK = base + Plan::kOffK;
  const uint32_t sV = base + Plan::kOffV;
  const uint32_t bar0 = base + Plan::kOffBar;
  auto q_full = [&](int i) { return bar0 + 8u * i; };
  auto k_full = [&](int s) { return bar0 + 8u * (kAttnQTiles + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (kAttnQTiles + KS + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (kAttnQTiles + 2 * KS + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (kAttnQTiles + 3 * KS + s); };
  auto s_full = [&](int i) { return bar0 + 8u * (Plan::kRingBars + i); };
  // P of slot i, keys 64 h .. 64 h + 63, in both CTAs' TMEM (leader's barrier).
  auto p_full = [&](int i, int h) { return bar0 + 8u * (Plan::kRingBars + kAttnQTiles + 2 * i + h); };
  auto o_full = [&](int i) { return bar0 + 8u * (Plan::kRingBars + 3 * kAttnQTiles + i); };
  const uint32_t drain = bar0 + 8u * (Plan::kRingBars + 4 * kAttnQTiles);  // every MMA issued has completed
  volatile uint32_t* tmem_holder = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffTmemHolder);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const uint32_t rank = cluster_ctarank();  // 0 = MMA leader of the pair
  const int group = (int)gridDim.y - 1 - (int)blockIdx.y;
  const int head = (int)(blockIdx.x >> 1) % p.heads;
  const int bat = (int)(blockIdx.x >> 1) / p.heads;
  const int kv_tiles_all = (p.seq_len + kAttnBKV - 1) / kAttnBKV;
  auto kv_tiles = [&](int qt) {
    return qt >= p.num_q_tiles ? 0 : (p.causal ? min(qt + 1, kv_tiles_all) : kv_tiles_all);
  };
  // This CTA's query tile in slot i, and the key tiles slot i runs (the
  // longer of the two CTAs' tiles; 0 when both are past the end).
  int qt_of[kAttnQTiles], n_of[kAttnQTiles];
#pragma unroll
  for (int i = 0; i < kAttnQTiles; ++i) {
    qt_of[i] = 4 * group + 2 * i + (int)rank;
    n_of[i] = max(kv_tiles(4 * group + 2 * i), kv_tiles(4 * group + 2 * i + 1));
  }
  const int n_max = max(n_of[0], n_of[1]);
  const int col0 = head * kAttnD;
  const int kv_col0 = (head / p.group) * kAttnD;

  if (warp == kAttnProducerWarp && lane == 0) {
    for (int i = 0; i < kAttnQTiles; ++i) {
      mbar_init(q_full(i), 1);     // leader's arrive + both CTAs' bytes
      mbar_init(s_full(i), 1);     // one commit from the leader's MMA thread
      mbar_init(p_full(i, 0), 8);  // four softmax warps of each CTA
      mbar_init(p_full(i, 1), 8);
      mbar_init(o_full(i), 1);
    }
    for (int s = 0; s < KS; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    mbar_init(drain, 1);
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == kAttnMmaWarp) {
    tmem_alloc_pair(smem_u32(const_cast<uint32_t*>(tmem_holder)), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barriers of both CTAs initialised before any remote arrive / transaction
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;  // S_i at columns 128 i, O_i at 256 + 128 i
  pdl_launch_dependents();
  pdl_wait();

  if (warp >= kAttnProducerWarp) {
    setmaxnreg_dec<kAttnRegsOther>();
    if (warp == kAttnProducerWarp) {
      // ---- TMA producer (both CTAs; completion on the leader's barriers) -------
      if (lane == 0) {
        const uint64_t pol_keep = l2_policy_evict_last();
        const uint64_t pol_once = l2_policy_evict_first();
        for (int i = 0; i < kAttnQTiles; ++i) {
          if (n_of[i] == 0) continue;
          if (rank == 0) mbar_arrive_expect_tx(q_full(i), 2 * Plan::kTileBytes);
          const uint32_t qb = mapa_shared(q_full(i), 0);
          for (int h = 0; h < 2; ++h) {
            tma_load_3d_pair(sQ + i * Plan::kTileBytes + h * 16384, &tmQ, qb, col0 + 64 * h, qt_of[i] * kAttnBQ, bat,
                             pol_once);
          }
        }
        bool ok = true;
        int issued = 0;
        for (int j = 0; j < n_max && ok; ++j) {
          const int s = j % KS;
          const uint32_t ph = (uint32_t)(j / KS) & 1u;
          if (!mbar_wait(k_empty(s), ph ^ 1u, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(k_full(s), 2 * Plan::kHalfBytes);
          const uint32_t kb = mapa_shared(k_full(s), 0);
          // Keys 64 rank .. 64 rank + 63 of the tile, as two [64 keys][64 d] atoms.
          for (int h = 0; h < 2; ++h) {
            tma_load_3d_pair(sK + s * Plan::kHalfBytes + h * 8192, &tmK, kb, kv_col0 + 64 * h,
                             j * kAttnBKV + 64 * (int)rank, bat, pol_keep);
          }
          if (!mbar_wait(v_empty(s), ph ^ 1u, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(v_full(s), 2 * Plan::kHalfBytes);
          const uint32_t vb = mapa_shared(v_full(s), 0);
          // Head columns 64 rank .. 64 rank + 63 of all 128 keys, as two
          // [64 keys][64 d] atoms (keys 0-63, 64-127).
          for (int hk = 0; hk < 2; ++hk) {
            tma_load_3d_pair(sV + s * Plan::kHalfBytes + hk * 8192, &tmV, vb, kv_col0 + 64 * (int)rank,
                             j * kAttnBKV + 64 * hk, bat, pol_keep);
          }
          ++issued;
        }
        if (!ok) attn_raise(p, abort_flag, kDevTimeoutProducer);
        // Drain (leader): its full barriers count both CTAs' bytes, so once the
        // latest phase of each has completed nothing of the pair is in flight.
        // The follower's loads are covered by this wait and the teardown
        // cluster barrier.
        if (rank == 0) {
          bool drained = true;
          for (int i = 0; drained && i < kAttnQTiles; ++i) {
            if (n_of[i] > 0) drained = mbar_wait(q_full(i), 0u, p.timeout_ns, nullptr);
          }
          for (int j = issued - 1; drained && j >= 0 && j >= issued - KS; --j) {
            drained = mbar_wait(k_full(j % KS), (uint32_t)(j / KS) & 1u, p.timeout_ns, nullptr) &&
                      mbar_wait(v_full(j % KS), (uint32_t)(j / KS) & 1u, p.timeout_ns, nullptr);
          }
          if (!drained) attn_raise(p, abort_flag, kDevTimeoutDrain);
        }
      }
      __syncwarp();
    } else if (warp == kAttnMmaWarp) {
      // ---- MMA issuer (leader CTA only) -------------------------------------------
      if (lane == 0 && rank == 0) {
        constexpr uint32_t idesc_s = idesc_bf16_f32(2 * kAttnBQ, kAttnBKV, false, false);  // Q x K^T, K-major
        constexpr uint32_t idesc_o = idesc_bf16_f32(2 * kAttnBQ, kAttnD, false, true);     // P (TMEM) x V (MN-major)
        // 16-wide K slices.  Q: [128 rows][64 d] atoms 16 KiB apart, a slice
        // 32 B into each row.  K half: [64 keys][64 d] atoms 8 KiB apart.
        // V half (MN-major, N = this CTA's 64 head columns = one atom wide):
        // a slice is 16 keys = 2 KiB into a [64 keys][64 d] atom, atoms (keys
        // 0-63, 64-127) 8 KiB apart.  P in TMEM steps 8 columns (16 bf16).
        auto qdesc = [](uint32_t tile, int k) {
          return smem_desc_sw128(tile + (uint32_t)((k >> 2) * 16384 + (k & 3) * 32), 16, 1024);
        };
        auto kdesc = [](uint32_t half, int k) {
          return smem_desc_sw128(half + (uint32_t)((k >> 2) * 8192 + (k & 3) * 32), 16, 1024);
        };
        auto vdesc = [](uint32_t half, int k) {
          return smem_desc_sw128(half + (uint32_t)((k >> 2) * 8192 + (k & 3) * 2048), 8192, 1024);
        };
        auto issue_s = [&](int i, int j) {
          const uint32_t qa = sQ + (uint32_t)(i * Plan::kTileBytes);
          const uint32_t kt = sK + (uint32_t)((j % KS) * Plan::kHalfBytes);
#pragma unroll
          for (int k = 0; k < kAttnD / kUmmaK; ++k) {
            umma_bf16_pair(tmem_base + (uint32_t)(i * 128), qdesc(qa, k), kdesc(kt, k), idesc_s, k > 0 ? 1u : 0u);
          }
        };
        auto issue_pv = [&](int i, int j, int h) {
          const uint32_t vt = sV + (uint32_t)((j % KS) * Plan::kHalfBytes);
#pragma unroll
          for (int k = 4 * h; k < 4 * h + 4; ++k) {
            umma_bf16_ts_pair(tmem_base + 256u + (uint32_t)(i * 128), tmem_base + (uint32_t)(i * 128 + k * 8),
                              vdesc(vt, k), idesc_o, (j > 0 || k > 0) ? 1u : 0u);
          }
        };
        auto wait_k = [&](int j) {
          return mbar_wait(k_full(j % KS), (uint32_t)(j / KS) & 1u, p.timeout_ns, abort_flag);
        };
        bool ok = true;
        for (int i = 0; ok && i < kAttnQTiles; ++i) {
          if (n_of[i] > 0) ok = mbar_wait(q_full(i), 0u, p.timeout_ns, abort_flag);
        }
        if (ok && n_max > 0) {
          ok = wait_k(0);
          if (ok) {
            tc_fence_after();
            for (int i = 0; i < kAttnQTiles; ++i) {
              if (n_of[i] == 0) continue;
              issue_s(i, 0);
              umma_commit_pair_both(s_full(i));
            }
            umma_commit_pair_both(k_empty(0));
          }
        }
        for (int j = 0; j < n_max && ok; ++j) {
          if (!mbar_wait(v_full(j % KS), (uint32_t)(j / KS) & 1u, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          bool k_ready = false;
#pragma unroll
          for (int i = 0; i < kAttnQTiles; ++i) {
            if (!ok || j >= n_of[i]) continue;
            if (!mbar_wait(p_full(i, 0), (uint32_t)j & 1u, p.timeout_ns, abort_flag)) {
              ok = false;
              continue;
            }
            tc_fence_after();
            issue_pv(i, j, 0);
            if (!mbar_wait(p_full(i, 1), (uint32_t)j & 1u, p.timeout_ns, abort_flag)) {
              ok = false;
              continue;
            }
            tc_fence_after();
            issue_pv(i, j, 1);
            if (i == kAttnQTiles - 1 || j >= n_of[kAttnQTiles - 1]) umma_commit_pair_both(v_empty(j % KS));
            if (j + 1 < n_of[i]) {
              if (!k_ready) {
                if (!wait_k(j + 1)) {
                  ok = false;
                  continue;
                }
                k_ready = true;
                tc_fence_after();
              }
              issue_s(i, j + 1);
              umma_commit_pair_both(s_full(i));
            } else {
              umma_commit_pair_both(o_full(i));
            }
          }
          if (ok && j + 1 < n_max) umma_commit_pair_both(k_empty((j + 1) % KS));
        }
        if (!ok) attn_raise(p, abort_flag, kDevTimeoutMma);
        umma_commit_pair(mapa_shared(drain, 0));
        if (!mbar_wait(drain, 0u, p.timeout_ns, nullptr)) attn_raise(p, abort_flag, kDevTimeoutDrain);
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kAttnRegsSoftmax>();
    // ---- softmax + epilogue of this CTA's rows (warps 0..3: slot 0, 4..7: slot 1) ----
    const int tile = warp >> 2;
    const int qw = warp & 3;
    const int row = qw * 32 + (int)lane;
    const int qt = qt_of[tile];
    const int n_kv = n_of[tile];
    const int q_idx = qt * kAttnBQ + row;
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + (uint32_t)(tile * 128);
    const uint32_t tO = tmem_base + lane_off + 256u + (uint32_t)(tile * 128);
    float m = -INFINITY;
    float l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const bool got = mbar_wait(s_full(tile), (uint32_t)j & 1u, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[kAttnBKV];
      {
        uint32_t r[4][32];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(tS + (uint32_t)(c * 32), r[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_wait_regs(r[c]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(r[c][i]);
        }
      }
      const int kv0 = j * kAttnBKV;
      // The diagonal tile, a tile past the sequence end, and the one extra
      // tile the shorter tile of a slot runs (all of it above the diagonal).
      const bool diag = p.causal && kv0 + kAttnBKV > qt * kAttnBQ;
      const bool masked = diag || kv0 + kAttnBKV > p.seq_len;
      if (masked) {
        const int lim = min(p.seq_len - kv0, diag ? q_idx - kv0 + 1 : kAttnBKV);
#pragma unroll
        for (int c = 0; c < kAttnBKV; ++c) x[c] = c < lim ? x[c] : -INFINITY;
      }
      float mxs[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxs[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < kAttnBKV; c += 2) mxs[(c >> 1) & 7] = max3f(mxs[(c >> 1) & 7], x[c], x[c + 1]);
      const float mx = max3f(max3f(mxs[0], mxs[1], mxs[2]), max3f(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]));
      const float m_new = fmaxf(m, mx * p.scale_log2);
      const bool move = (m == -INFINITY) ? (m_new != -INFINITY) : (m_new > m + kAttnRescaleLog2);
      const float factor = (move && m != -INFINITY) ? fast_exp2(m - m_new) : 1.0f;
      const float m_next = move ? m_new : m;
      const float m_use = (m_next == -INFINITY) ? 0.0f : m_next;
      if (j > 0 && __any_sync(0xffffffffu, move && factor != 1.0f)) {
        // S_i(j) was issued after P_i(j-1) V(j-1) and its completion signal
        // covers that product: O is stable until this CTA's P is in.
        uint32_t r[32];
#pragma unroll 1
        for (int c = 0; c < kAttnD / 32; ++c) {
          const uint32_t ta = tO + (uint32_t)(c * 32);
          tmem_ld_32x32b_x32(ta, r);
          tmem_ld_wait_regs(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
          tmem_st_32x32b_x32(ta, r);
        }
      }
      if (move) {
        l *= factor;
        m = m_new;
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pw[32];
        l += masked ? row_exp<64, false>(x + 64 * h, p.scale_log2, m_use, pw)
                    : row_exp<64, true>(x + 64 * h, p.scale_log2, m_use, pw);
        tmem_st_32x32b_x32(tS + (uint32_t)(32 * h), pw);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(mapa_shared(p_full(tile, h), 0));
      }
    }
    if (!ok) {
      if (lane == 0) attn_raise(p, abort_flag, kDevTimeoutEpilogue);
    } else if (n_kv > 0) {
      const bool last = mbar_wait(o_full(tile), 0u, p.timeout_ns, abort_flag);
      if (__all_sync(0xffffffffu, last)) {
        // Rows past the end of the sequence are neither needed nor stored (a
        // whole tile past the end makes no store at all).
        if (qt * kAttnBQ + qw * 32 < p.seq_len) {
          tc_fence_after();
          const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
          const uint32_t stage = sQ + (uint32_t)(tile * Plan::kTileBytes + qw * 8192);
#pragma unroll 1
          for (int half = 0; half < 2; ++half) {
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(tO + (uint32_t)(half * 64), lo);
            tmem_ld_32x32b_x32(tO + (uint32_t)(half * 64 + 32), hi);
            tmem_ld_wait_regs(lo);
            tmem_ld_wait_regs(hi);
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              lo[i] = __float_as_uint(__uint_as_float(lo[i]) * inv_l);
              hi[i] = __float_as_uint(__uint_as_float(hi[i]) * inv_l);
            }
            stage_row64(lo, hi, false, stage + (uint32_t)(half * 4096), 0u, lane);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            for (int half = 0; half < 2; ++half) {
              tma_store_3d(&tmO, stage + (uint32_t)(half * 4096), col0 + 64 * half, qt * kAttnBQ + qw * 32, bat);
            }
            bulk_commit_group();
            bulk_wait_group_read<0>();
          }
          __syncwarp();
        }
      } else if (lane == 0) {
        attn_raise(p, abort_flag, kDevTimeoutEpilogue);
      }
    }
  }

  // ---- teardown -------------------------------------------------------------
  tc_fence_before();
  cluster_sync_all();  // no CTA leaves while its peer may still touch its barriers, smem or TMEM
  if (warp == kAttnMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 512);
  }
#endif  // B200_NO_SM100A_FEATURES
}

}  // namespace b200
