// Flash attention forward for sm_100a (tcgen05 + TMEM + TMA), the reference's
// flash_attn operator (flash_attn/flash_attn.cpp:5-30, fa2_tma_lazy_rescale.cu):
// O = softmax(Q K^T / sqrt(D)) V, optionally causal, bf16 in and out, fp32
// softmax statistics and accumulation, Q/O stored [batch, seq, heads, 128] and
// K/V [batch, seq, kv_heads, 128]; query head h reads key/value head
// h / (heads / kv_heads) (grouped-query attention, as the reference's kernel,
// fa2_tma_lazy_rescale.cu:113-114).
//
// One CTA per (128 query rows, head, batch); 192 threads:
//   warp 0      TMA producer: the Q tile once, then K and V tiles of 128 keys
//               through a 2-deep ring each;
//   warp 1      TMEM owner and single-thread tcgen05.mma issuer:
//                 S_j = Q K_j^T   into TMEM (two buffers, S_{j+1} is computed
//                                 while the softmax works on S_j),
//                 O  += P_j V_j   into TMEM (A = P from shared memory,
//                                 B = V tile in its natural [key][d] layout,
//                                 i.e. an MN-major operand);
//   warps 2..5  softmax, one thread per query row (= TMEM lane): S row from
//               TMEM, running max and sum in fp32 (exp2 domain), P row as
//               bf16 into 128B-swizzled shared memory; lazy rescaling — the
//               running max, and with it O in TMEM, is only moved when the row
//               max grows by more than 2^8 — and at the end O / l -> bf16 ->
//               TMA store.
// Every wait is bounded (status bits on expiry), as in the GEMM kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "gemm_sm100.cuh"
#include "ptx_sm100.cuh"

namespace b200 {

constexpr int kAttnD = 128;      // head dimension
constexpr int kAttnBQ = 128;     // query rows per CTA (UMMA M, TMEM lanes)
constexpr int kAttnBKV = 128;    // keys per tile
constexpr int kAttnStages = 2;   // K and V ring depth
constexpr float kAttnRescaleLog2 = 8.0f;  // lazy rescale threshold (P stays <= 2^8)

struct AttnParams {
  int32_t seq_len, heads, batch;
  int32_t group;  // heads / kv_heads: query heads per key/value head
  int32_t num_q_tiles;
  uint32_t causal;
  float scale_log2;  // log2(e) / sqrt(D): scores go straight to the exp2 domain
  uint64_t timeout_ns;
  uint32_t* status;
};

struct AttnSmemPlan {
  static constexpr int kTileBytes = 128 * 128 * 2;  // any 128 x 128 bf16 tile: 32 KiB
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kTileBytes;
  static constexpr int kOffV = kOffK + kAttnStages * kTileBytes;
  static constexpr int kOffP = kOffV + kAttnStages * kTileBytes;  // P, then the O staging at the end
  static constexpr int kOffBar = kOffP + kTileBytes;
  // q_full, k_full[S], k_empty[S], v_full[S], v_empty[S], s_full[2], s_empty[2], p_full, o_done, drain
  static constexpr int kNumBars = 1 + 4 * kAttnStages + 4 + 3;
  static constexpr int kOffTmemHolder = kOffBar + kNumBars * 8;
  static constexpr int kOffAbort = kOffTmemHolder + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAllocBytes = kBytes + 1024;
  static_assert(kAllocBytes <= 232448, "attention shared memory plan exceeds 227 KiB");
};

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void attn_raise(const AttnParams& p, volatile uint32_t* abort_flag, uint32_t code) {
  *abort_flag = 1u;
  if (p.status != nullptr) atomicOr(p.status, code);
}

// Grid (num_q_tiles, heads, batch).  Query tiles are taken in reverse order so
// that, with a causal mask, the longest rows start first.
__global__ void __launch_bounds__(kNumThreads, 1)
    flash_attn_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                          const __grid_constant__ AttnParams p) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, (uint32_t)kDevWrongArch);
#else
  using Plan = AttnSmemPlan;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_u32 = smem_u32(smem_raw);
  const uint32_t base = (raw_u32 + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_u32);
  const uint32_t sQ = base + Plan::kOffQ;
  const uint32_t sK = base + Plan::kOffK;
  const uint32_t sV = base + Plan::kOffV;
  const uint32_t sP = base + Plan::kOffP;
  const uint32_t bar0 = base + Plan::kOffBar;
  const uint32_t q_full = bar0;
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (1 + kAttnStages + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + 2 * kAttnStages + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (1 + 3 * kAttnStages + s); };
  auto s_full = [&](int b) { return bar0 + 8u * (1 + 4 * kAttnStages + b); };
  auto s_empty = [&](int b) { return bar0 + 8u * (3 + 4 * kAttnStages + b); };
  const uint32_t p_full = bar0 + 8u * (5 + 4 * kAttnStages);
  const uint32_t o_done = p_full + 8u;
  const uint32_t drain = o_done + 8u;  // every MMA issued has completed (teardown)
  volatile uint32_t* tmem_holder = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffTmemHolder);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  const int qt = p.num_q_tiles - 1 - (int)blockIdx.x;
  const int head = blockIdx.y;
  const int bat = blockIdx.z;
  const int kv_tiles_all = (p.seq_len + kAttnBKV - 1) / kAttnBKV;
  const int n_kv = p.causal ? min(qt + 1, kv_tiles_all) : kv_tiles_all;
  const int col0 = head * kAttnD;  // column of this head in the [seq, heads * D] view
  const int kv_col0 = (head / p.group) * kAttnD;  // its key/value head in [seq, kv_heads * D]

  if (warp == 0 && lane == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAttnStages; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
      mbar_init(v_full(s), 1);
      mbar_init(v_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(s_full(b), 1);
      mbar_init(s_empty(b), kEpiWarps);
    }
    mbar_init(p_full, kEpiWarps);
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmO);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_holder)), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;  // S buffers at columns 0 and 128, O at 256
  pdl_launch_dependents();
  pdl_wait();

  if (warp == 0) {
    // ---- TMA producer ------------------------------------------------------
    if (lane == 0) {
      const uint64_t pol_keep = l2_policy_evict_last();  // K, V: read by every query tile of the head
      const uint64_t pol_once = l2_policy_evict_first();  // Q: read once
      mbar_arrive_expect_tx(q_full, Plan::kTileBytes);
      for (int i = 0; i < 2; ++i) tma_load_3d(sQ + i * 16384, &tmQ, q_full, col0 + 64 * i, qt * kAttnBQ, bat, pol_once);
      bool ok = true;
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(k_empty(s), ph ^ 1u, p.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(k_full(s), Plan::kTileBytes);
        for (int i = 0; i < 2; ++i) {
          tma_load_3d(sK + s * Plan::kTileBytes + i * 16384, &tmK, k_full(s), kv_col0 + 64 * i, j * kAttnBKV, bat,
                      pol_keep);
        }
        ++k_issued;
        if (!mbar_wait(v_empty(s), ph ^ 1u, p.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(v_full(s), Plan::kTileBytes);
        // V tile as two 64-key halves, each two 64-column atoms of [64 keys][64 d].
        for (int hk = 0; hk < 2; ++hk) {
          for (int i = 0; i < 2; ++i) {
            tma_load_3d(sV + s * Plan::kTileBytes + hk * 16384 + i * 8192, &tmV, v_full(s), kv_col0 + 64 * i,
                        j * kAttnBKV + 64 * hk, bat, pol_keep);
          }
        }
        ++v_issued;
      }
      if (!ok) attn_raise(p, abort_flag, kDevTimeoutProducer);
      // Let the copies in flight land before the CTA can leave.
      if (!mbar_wait(q_full, 0u, p.timeout_ns, nullptr)) attn_raise(p, abort_flag, kDevTimeoutDrain);
      bool drained = true;
      for (int j = k_issued - 1; drained && j >= 0 && j >= k_issued - kAttnStages; --j) {
        drained = mbar_wait(k_full(j & 1), (uint32_t)(j >> 1) & 1u, p.timeout_ns, nullptr);
      }
      for (int j = v_issued - 1; drained && j >= 0 && j >= v_issued - kAttnStages; --j) {
        drained = mbar_wait(v_full(j & 1), (uint32_t)(j >> 1) & 1u, p.timeout_ns, nullptr);
      }
      if (!drained) attn_raise(p, abort_flag, kDevTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer ----------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(kAttnBQ, kAttnBKV, false, false);  // Q (K-major) x K^T (K-major)
      constexpr uint32_t idesc_o = idesc_bf16_f32(kAttnBQ, kAttnD, false, true);     // P (K-major) x V (MN-major)
      // 16-wide K slices: K-major operands step 32 B inside a 64-wide atom
      // and 16 KiB between the two atoms; the MN-major V steps 16 keys =
      // 2 KiB inside a 64-key half and 16 KiB between halves.
      auto kmajor = [](uint32_t tile, int k) {
        return smem_desc_sw128(tile + (uint32_t)((k >> 2) * 16384 + (k & 3) * 32), 16, 1024);
      };
      auto vdesc = [](uint32_t tile, int k) {
        return smem_desc_sw128(tile + (uint32_t)((k >> 2) * 16384 + (k & 3) * 2048), 8192, 1024);
      };
      bool ok = mbar_wait(q_full, 0u, p.timeout_ns, abort_flag);
      auto pv = [&](int i) {
        if (!ok) return;
        if (!mbar_wait(p_full, (uint32_t)i & 1u, p.timeout_ns, abort_flag) ||
            !mbar_wait(v_full(i & 1), (uint32_t)(i >> 1) & 1u, p.timeout_ns, abort_flag)) {
          ok = false;
          return;
        }
        tc_fence_after();
        const uint32_t vt = sV + (uint32_t)((i & 1) * Plan::kTileBytes);
#pragma unroll
        for (int k = 0; k < kAttnBKV / kUmmaK; ++k) {
          umma_bf16(tmem_base + 256u, kmajor(sP, k), vdesc(vt, k), idesc_o, (i > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(v_empty(i & 1));
        umma_commit(o_done);
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int s = j & 1;
        const uint32_t ph = (uint32_t)(j >> 1) & 1u;
        if (!mbar_wait(k_full(s), ph, p.timeout_ns, abort_flag) ||
            !mbar_wait(s_empty(s), ph ^ 1u, p.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kt = sK + (uint32_t)(s * Plan::kTileBytes);
#pragma unroll
        for (int k = 0; k < kAttnD / kUmmaK; ++k) {
          umma_bf16(tmem_base + (uint32_t)(s * kAttnBKV), kmajor(sQ, k), kmajor(kt, k), idesc_s, k > 0 ? 1u : 0u);
        }
        umma_commit(k_empty(s));
        umma_commit(s_full(s));
        if (j >= 1) pv(j - 1);
      }
      if (ok && n_kv > 0) pv(n_kv - 1);
      if (!ok) attn_raise(p, abort_flag, kDevTimeoutMma);
      umma_commit(drain);
      if (!mbar_wait(drain, 0u, p.timeout_ns, nullptr)) attn_raise(p, abort_flag, kDevTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ---- softmax + epilogue (warps 2..5) -------------------------------------
    const int qw = warp & 3;                // TMEM lane quarter this warp may access
    const int row = qw * 32 + (int)lane;     // query row in the tile
    const int q_idx = qt * kAttnBQ + row;    // query position
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    float m = -INFINITY;  // running max (exp2 domain) the stored P and O refer to
    float l = 0.0f;       // running sum of P
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      const uint32_t ph = (uint32_t)(j >> 1) & 1u;
      const bool got = mbar_wait(s_full(s), ph, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float x[kAttnBKV];
      {
        uint32_t r[32];
#pragma unroll
        for (int c = 0; c < kAttnBKV / 32; ++c) {
          tmem_ld_32x32b_x32(tmem_base + lane_off + (uint32_t)(s * kAttnBKV + c * 32), r);
          tmem_ld_wait_regs(r);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(r[i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty(s));  // S buffer s may be overwritten by S_{j+2}
      const int kv0 = j * kAttnBKV;
      const bool diag = p.causal && kv0 + kAttnBKV > qt * kAttnBQ;  // the tile crossing the diagonal
      // Scale into the exp2 domain and take the row max.  Eight independent
      // partial maxima (and sums below): one thread owns the whole row, so a
      // single dependency chain over 128 keys would serialise on latency.
      // Only the diagonal tile and a tile past the sequence end need masks:
      // keys c >= lim are masked.
      const bool masked = diag || kv0 + kAttnBKV > p.seq_len;
      const int lim = min(p.seq_len - kv0, diag ? q_idx - kv0 + 1 : kAttnBKV);
      float mxs[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxs[i] = -INFINITY;
      if (!masked) {
#pragma unroll
        for (int c = 0; c < kAttnBKV; ++c) {
          x[c] *= p.scale_log2;
          mxs[c & 7] = fmaxf(mxs[c & 7], x[c]);
        }
      } else {
#pragma unroll
        for (int c = 0; c < kAttnBKV; ++c) {
          x[c] = c < lim ? x[c] * p.scale_log2 : -INFINITY;
          mxs[c & 7] = fmaxf(mxs[c & 7], x[c]);
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mxs[0], mxs[1]), fmaxf(mxs[2], mxs[3])),
                             fmaxf(fmaxf(mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7])));
      const float m_new = fmaxf(m, mx);
      // Move the reference max only when the row max grew by more than 2^8
      // (or nothing was seen yet): P stays below 2^8, and O is rescaled rarely.
      const bool move = (m == -INFINITY) ? (m_new != -INFINITY) : (m_new > m + kAttnRescaleLog2);
      const float factor = (move && m != -INFINITY) ? fast_exp2(m - m_new) : 1.0f;
      // P and its row sum with the max the row will use from now on — all
      // before waiting for the previous P V product, so the exponentials
      // overlap that MMA; P is kept packed as bf16 pairs.
      const float m_next = move ? m_new : m;
      const float m_use = (m_next == -INFINITY) ? 0.0f : m_next;
      float sums[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sums[i] = 0.0f;
      uint32_t pw[kAttnBKV / 2];
#pragma unroll
      for (int c = 0; c < kAttnBKV; c += 2) {
        // exp2(-inf) is +0: masked keys need no test.
        const float e0 = fast_exp2(x[c] - m_use);
        const float e1 = fast_exp2(x[c + 1] - m_use);
        sums[(c >> 1) & 7] += e0 + e1;
        __nv_bfloat162 h = __floats2bfloat162_rn(e0, e1);
        pw[c / 2] = *reinterpret_cast<uint32_t*>(&h);
      }
      const float sum = ((sums[0] + sums[1]) + (sums[2] + sums[3])) + ((sums[4] + sums[5]) + (sums[6] + sums[7]));
      if (j > 0) {
        // P_{j-1} V_{j-1} done: the P buffer is free and O is stable.
        const bool prev = mbar_wait(o_done, (uint32_t)(j - 1) & 1u, p.timeout_ns, abort_flag);
        if (!__all_sync(0xffffffffu, prev)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, move && factor != 1.0f)) {
          uint32_t r[32];
#pragma unroll 1
          for (int c = 0; c < kAttnD / 32; ++c) {
            const uint32_t ta = tmem_base + lane_off + 256u + (uint32_t)(c * 32);
            tmem_ld_32x32b_x32(ta, r);
            tmem_ld_wait_regs(r);
#pragma unroll
            for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) * factor);
            tmem_st_32x32b_x32(ta, r);
          }
          tmem_st_wait();
        }
      }
      if (move) {
        l *= factor;
        m = m_new;
      }
      l += sum;
      // P row -> shared memory, bf16, 128B-swizzled K-major (keys contiguous):
      // two atoms of 64 keys, 16-byte chunk c of row r at chunk c ^ (r & 7).
#pragma unroll
      for (int a = 0; a < 2; ++a) {
        const uint32_t row_addr = sP + (uint32_t)(a * 16384 + row * 128);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const int w0 = a * 32 + cc * 4;
          const uint32_t dst = row_addr + (((uint32_t)cc ^ ((uint32_t)row & 7u)) << 4);
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(pw[w0]), "r"(pw[w0 + 1]),
                       "r"(pw[w0 + 2]), "r"(pw[w0 + 3])
                       : "memory");
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (!ok) {
      if (lane == 0) attn_raise(p, abort_flag, kDevTimeoutEpilogue);
    } else if (n_kv > 0) {
      // O / l -> bf16 -> TMA store, through this warp's 8 KiB of the (now
      // idle) P buffer: two [32 rows][64 d] swizzled chunks.
      const bool last = mbar_wait(o_done, (uint32_t)(n_kv - 1) & 1u, p.timeout_ns, abort_flag);
      if (__all_sync(0xffffffffu, last)) {
        tc_fence_after();
        const float inv_l = l > 0.0f ? 1.0f / l : 0.0f;
        const uint32_t stage = sP + (uint32_t)(qw * 8192);
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          uint32_t lo[32], hi[32];
          tmem_ld_32x32b_x32(tmem_base + lane_off + 256u + (uint32_t)(half * 64), lo);
          tmem_ld_32x32b_x32(tmem_base + lane_off + 256u + (uint32_t)(half * 64 + 32), hi);
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
      } else if (lane == 0) {
        attn_raise(p, abort_flag, kDevTimeoutEpilogue);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
#endif  // B200_NO_SM100A_FEATURES
}

}  // namespace b200
