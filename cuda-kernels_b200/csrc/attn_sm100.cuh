// Flash attention forward for sm_100a (tcgen05 + TMEM + TMA), the reference's
// flash_attn operator (flash_attn/flash_attn.cpp:5-30, fa2_tma_lazy_rescale.cu):
// O = softmax(Q K^T / sqrt(D)) V, optionally causal, bf16 in and out, fp32
// softmax statistics and accumulation, Q/O stored [batch, seq, heads, 128] and
// K/V [batch, seq, kv_heads, 128]; query head h reads key/value head
// h / (heads / kv_heads) (grouped-query attention, as the reference's kernel,
// fa2_tma_lazy_rescale.cu:113-114).
//
// One CTA per (two 128-row query tiles, head, batch); 384 threads in three
// warpgroups:
//   warps 0..3  softmax of query tile 0, warps 4..7 of tile 1 (below);
//   warp 8      TMA producer: both Q tiles once, then K and V tiles of 128
//               keys through a 2-deep ring each (each K and V tile serves both
//               query tiles);
//   warp 9      TMEM owner and single-thread tcgen05.mma issuer, for query
//               tile i = 0, 1:
//                 S_i  = Q_i K_j^T  into TMEM columns [128 i, 128 i + 128),
//                 O_i += P_i V_j    into TMEM columns [256 + 128 i, ...), A = P_i
//                                   read from TMEM, where the softmax wrote it
//                                   (bf16) over S_i, B = the V tile in its
//                                   natural [key][d] layout (an MN-major operand);
//               issued in the order P_0 V_j, S_0 (j+1), P_1 V_j, S_1 (j+1)
//               (P V as two halves of 64 keys, each after its half of P), so
//               that each softmax warpgroup works while the tensor cores run
//               the other tile's two products;
//   warps 10,11 idle.
// Softmax: one thread per query row (= TMEM lane) holds the row's 128 scores
// in registers (the third warpgroup gives up registers with setmaxnreg so
// that the softmax warpgroups have 208 each): S row from TMEM, running max and
// sum in fp32 (exp2 domain), P row as bf16 back into TMEM in two 64-key
// halves (the first half of P V starts while the second is computed); lazy rescaling —
// the running max, and with it O in TMEM, is only moved when the row max grows
// by more than 2^8 — and at the end O / l -> bf16 -> TMA store (staged in the
// tile's Q buffer).
// The exponentials run on the MUFU unit (16 per clock per SM, as long as the
// tile's MMAs); poly_exp2x2 can move a share of them to the FMA pipe
// (kAttnPolyEvery).
// Every wait is bounded (status bits on expiry), as in the GEMM kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "gemm_sm100.cuh"
#include "ptx_sm100.cuh"

namespace b200 {

constexpr int kAttnD = 128;      // head dimension
constexpr int kAttnBQ = 128;     // query rows per tile (UMMA M, TMEM lanes)
constexpr int kAttnBKV = 128;    // keys per tile
constexpr int kAttnQTiles = 2;   // query tiles per CTA, one softmax warpgroup each
#ifndef B200_ATTN_K_STAGES
#define B200_ATTN_K_STAGES 2
#endif
#ifndef B200_ATTN_V_STAGES
#define B200_ATTN_V_STAGES 2
#endif
// K and V ring depths.  A third stage of either (the shared memory has room
// for one) measured the same on B200, with or without the softmax: the
// loads are not what the tensor pipe waits for.
constexpr int kAttnKStages = B200_ATTN_K_STAGES;
constexpr int kAttnVStages = B200_ATTN_V_STAGES;
constexpr int kAttnThreads = 128 * (kAttnQTiles + 1);
constexpr int kAttnProducerWarp = 4 * kAttnQTiles;
constexpr int kAttnMmaWarp = kAttnProducerWarp + 1;
// Registers per thread: at launch (the kernel is compiled to exactly this),
// after reallocation for the producer/MMA warpgroup and for the softmax
// warpgroups.  128 * 88 + 256 * 208 = 384 * 168.
constexpr uint32_t kAttnRegsLaunch = 168, kAttnRegsOther = 88, kAttnRegsSoftmax = 208;
static_assert(128 * kAttnRegsOther + kAttnQTiles * 128 * kAttnRegsSoftmax <= kAttnThreads * kAttnRegsLaunch,
              "register reallocation exceeds the launch pool");
// Every kAttnPolyEvery-th pair of exponentials on the FMA pipe (0: none).
// Measured on B200: every 4th pair cost 2 %, every 2nd 7 % (the softmax is
// bound by latency and issue, not by the MUFU rate), so it is off.  Neither
// did taking turns help (the two softmax warpgroups' exponential phases one
// after the other through an mbarrier, each with the MUFU to itself: 2-5 %
// slower), nor splitting each row over two warpgroups of 64 keys each (their
// maxima exchanged through shared memory: 7 % slower).
#ifndef B200_ATTN_POLY_EVERY
#define B200_ATTN_POLY_EVERY 0
#endif
constexpr int kAttnPolyEvery = B200_ATTN_POLY_EVERY;
constexpr float kAttnRescaleLog2 = 8.0f;  // lazy rescale threshold (P stays <= 2^8)

struct AttnParams {
  int32_t seq_len, heads, batch;
  int32_t group;  // heads / kv_heads: query heads per key/value head
  int32_t num_q_tiles;
  uint32_t causal;
  // Query tiles of CTA row y: 0 -> (2 (Y-1-y), 2 (Y-1-y) + 1), the longest
  // rows first; 1 -> (y, T-1-y), a short and a long causal row together, so
  // that every CTA carries the same work (used when the grid is one wave).
  uint32_t balanced;
  float scale_log2;  // log2(e) / sqrt(D): scores go straight to the exp2 domain
  uint64_t timeout_ns;
  uint32_t* status;
};

struct AttnSmemPlan {
  static constexpr int kTileBytes = 128 * 128 * 2;  // any 128 x 128 bf16 tile: 32 KiB
  static constexpr int kOffQ = 0;                   // kAttnQTiles tiles; O staging at the end
  static constexpr int kOffK = kOffQ + kAttnQTiles * kTileBytes;
  static constexpr int kOffV = kOffK + kAttnKStages * kTileBytes;
  static constexpr int kOffBar = kOffV + kAttnVStages * kTileBytes;
  // q_full[Q], k_full[KS], k_empty[KS], v_full[VS], v_empty[VS], s_full[Q], p_full[Q][2], o_full[Q], drain
  static constexpr int kRingBars = kAttnQTiles + 2 * kAttnKStages + 2 * kAttnVStages;
  static constexpr int kNumBars = kRingBars + 4 * kAttnQTiles + 1;
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

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair, on the FMA pipe instead of the MUFU unit, for x <= 2^7
// (clamped below at -125 so the result stays a normal float; those values
// are below 2^-124 and vanish against the row sum, which is >= 1).
// x = n + f with n = rint(x) (adding 1.5 * 2^23 leaves rint(x) in the low
// mantissa bits) and |f| <= 1/2; 2^f from a cubic fitted for this build by
// Lawson's iteration to minimax relative error on [-1/2, 1/2] (7.5e-5,
// against the 2^-9 rounding of P to bf16); n is added into the exponent.
__device__ __forceinline__ float2 poly_exp2x2(float2 x) {
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 shift = make_float2(12582912.0f, 12582912.0f);
  const float2 t = __fadd2_rn(x, shift);
  const float2 n = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
  float2 y = __ffma2_rn(make_float2(0x1.c3f76p-5f, 0x1.c3f76p-5f), f, make_float2(0x1.f0de1cp-3f, 0x1.f0de1cp-3f));
  y = __ffma2_rn(y, f, make_float2(0x1.62f31ap-1f, 0x1.62f31ap-1f));
  y = __ffma2_rn(y, f, make_float2(0x1.fff692p-1f, 0x1.fff692p-1f));
  return make_float2(__uint_as_float(__float_as_uint(y.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(y.y) + (__float_as_uint(t.y) << 23)));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// P = 2^(x * scale - m_use) for N scores of one row, packed as bf16 pairs
// (key 2c in the low half of word c), and their sum.  kPoly: every
// kAttnPolyEvery-th pair goes through poly_exp2x2 (only for tiles without
// masked keys: there x = -inf must give exactly 0).
template <int N, bool kPoly>
__device__ __forceinline__ float row_exp(const float* x, float scale, float m_use, uint32_t (&pw)[N / 2]) {
  const float2 sc = make_float2(scale, scale);
  const float2 nm = make_float2(-m_use, -m_use);
  float2 acc[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int c = 0; c < N; c += 2) {
    const float2 t = __ffma2_rn(make_float2(x[c], x[c + 1]), sc, nm);
    float2 e;
    if (kPoly && kAttnPolyEvery > 0 && ((c >> 1) % (kAttnPolyEvery > 0 ? kAttnPolyEvery : 1)) == kAttnPolyEvery - 1) {
      e = poly_exp2x2(t);
    } else {
      e = make_float2(fast_exp2(t.x), fast_exp2(t.y));
    }
    acc[(c >> 1) & 3] = __fadd2_rn(acc[(c >> 1) & 3], e);
    pw[c >> 1] = pack_bf16x2(e.x, e.y);
  }
  const float2 s01 = __fadd2_rn(acc[0], acc[1]);
  const float2 s23 = __fadd2_rn(acc[2], acc[3]);
  const float2 s = __fadd2_rn(s01, s23);
  return s.x + s.y;
}

__device__ __forceinline__ void attn_raise(const AttnParams& p, volatile uint32_t* abort_flag, uint32_t code) {
  *abort_flag = 1u;
  if (p.status != nullptr) atomicOr(p.status, code);
}

// Grid (heads * batch, ceil(num_q_tiles / 2)).  Blocks start in linear
// order, x fastest, and query tile pairs are taken in reverse order of y: the
// longest causal rows of every head start first (longest-first scheduling).
__global__ void __launch_bounds__(kAttnThreads, 1)
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
  const uint32_t bar0 = base + Plan::kOffBar;
  auto q_full = [&](int i) { return bar0 + 8u * i; };
  auto k_full = [&](int s) { return bar0 + 8u * (kAttnQTiles + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (kAttnQTiles + kAttnKStages + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (kAttnQTiles + 2 * kAttnKStages + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (kAttnQTiles + 2 * kAttnKStages + kAttnVStages + s); };
  auto s_full = [&](int i) { return bar0 + 8u * (Plan::kRingBars + i); };
  // P of tile i, keys 64 h .. 64 h + 63, in TMEM.
  auto p_full = [&](int i, int h) { return bar0 + 8u * (Plan::kRingBars + kAttnQTiles + 2 * i + h); };
  auto o_full = [&](int i) { return bar0 + 8u * (Plan::kRingBars + 3 * kAttnQTiles + i); };
  const uint32_t drain = bar0 + 8u * (Plan::kRingBars + 4 * kAttnQTiles);  // every MMA issued has completed
  // Ring slot and phase parity of key tile j.
  auto k_slot = [](int j) { return j % kAttnKStages; };
  auto k_par = [](int j) { return (uint32_t)(j / kAttnKStages) & 1u; };
  auto v_slot = [](int j) { return j % kAttnVStages; };
  auto v_par = [](int j) { return (uint32_t)(j / kAttnVStages) & 1u; };
  volatile uint32_t* tmem_holder = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffTmemHolder);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;
  // The CTA's two query tiles: qt_of[1] >= qt_of[0] + 1 (or past the end).
  int qt_of[kAttnQTiles];
  if (p.balanced) {
    qt_of[0] = (int)blockIdx.y;
    qt_of[1] = p.num_q_tiles - 1 - (int)blockIdx.y;
    if (qt_of[1] <= qt_of[0]) qt_of[1] = p.num_q_tiles;  // the middle tile of an odd count stays alone
  } else {
    qt_of[0] = kAttnQTiles * ((int)gridDim.y - 1 - (int)blockIdx.y);
    qt_of[1] = qt_of[0] + 1;
  }
  const int head = (int)blockIdx.x % p.heads;
  const int bat = (int)blockIdx.x / p.heads;
  const int kv_tiles_all = (p.seq_len + kAttnBKV - 1) / kAttnBKV;
  // Key tiles query tile qt reads (the causal mask ends at the diagonal tile);
  // 0 for a second tile past the end of the sequence.
  auto kv_tiles = [&](int qt) {
    return qt >= p.num_q_tiles ? 0 : (p.causal ? min(qt + 1, kv_tiles_all) : kv_tiles_all);
  };
  const int n0 = kv_tiles(qt_of[0]);
  const int n1 = kv_tiles(qt_of[1]);  // >= n0, or 0
  const int n_max = max(n0, n1);
  const int n_q = n1 > 0 ? 2 : 1;    // query tiles this CTA holds
  const int col0 = head * kAttnD;                  // column of this head in the [seq, heads * D] view
  const int kv_col0 = (head / p.group) * kAttnD;   // its key/value head in [seq, kv_heads * D]

  if (warp == kAttnProducerWarp && lane == 0) {
    for (int i = 0; i < kAttnQTiles; ++i) {
      mbar_init(q_full(i), 1);
      mbar_init(s_full(i), 1);
      mbar_init(p_full(i, 0), 4);
      mbar_init(p_full(i, 1), 4);
      mbar_init(o_full(i), 1);
    }
    for (int s = 0; s < kAttnKStages; ++s) {
      mbar_init(k_full(s), 1);
      mbar_init(k_empty(s), 1);
    }
    for (int s = 0; s < kAttnVStages; ++s) {
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
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_holder)), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;  // S_i at columns 128 i, O_i at 256 + 128 i
  pdl_launch_dependents();
  pdl_wait();

  if (warp >= kAttnProducerWarp) {
    setmaxnreg_dec<kAttnRegsOther>();
    if (warp == kAttnProducerWarp) {
      // ---- TMA producer ------------------------------------------------------
      if (lane == 0) {
        const uint64_t pol_keep = l2_policy_evict_last();  // K, V: read by every query tile of the head
        const uint64_t pol_once = l2_policy_evict_first();  // Q: read once
        for (int i = 0; i < n_q; ++i) {
          mbar_arrive_expect_tx(q_full(i), Plan::kTileBytes);
          for (int h = 0; h < 2; ++h) {
            tma_load_3d(sQ + i * Plan::kTileBytes + h * 16384, &tmQ, q_full(i), col0 + 64 * h,
                        qt_of[i] * kAttnBQ, bat, pol_once);
          }
        }
        bool ok = true;
        int k_issued = 0, v_issued = 0;
        for (int j = 0; j < n_max && ok; ++j) {
          const int sk = k_slot(j), sv = v_slot(j);
          if (!mbar_wait(k_empty(sk), k_par(j) ^ 1u, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(k_full(sk), Plan::kTileBytes);
          for (int h = 0; h < 2; ++h) {
            tma_load_3d(sK + sk * Plan::kTileBytes + h * 16384, &tmK, k_full(sk), kv_col0 + 64 * h, j * kAttnBKV,
                        bat, pol_keep);
          }
          ++k_issued;
          if (!mbar_wait(v_empty(sv), v_par(j) ^ 1u, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(v_full(sv), Plan::kTileBytes);
          // V tile as two 64-key halves, each two 64-column atoms of [64 keys][64 d].
          for (int hk = 0; hk < 2; ++hk) {
            for (int h = 0; h < 2; ++h) {
              tma_load_3d(sV + sv * Plan::kTileBytes + hk * 16384 + h * 8192, &tmV, v_full(sv), kv_col0 + 64 * h,
                          j * kAttnBKV + 64 * hk, bat, pol_keep);
            }
          }
          ++v_issued;
        }
        if (!ok) attn_raise(p, abort_flag, kDevTimeoutProducer);
        // Let the copies in flight land before the CTA can leave.
        bool drained = true;
        for (int i = 0; drained && i < n_q; ++i) drained = mbar_wait(q_full(i), 0u, p.timeout_ns, nullptr);
        for (int j = k_issued - 1; drained && j >= 0 && j >= k_issued - kAttnKStages; --j) {
          drained = mbar_wait(k_full(k_slot(j)), k_par(j), p.timeout_ns, nullptr);
        }
        for (int j = v_issued - 1; drained && j >= 0 && j >= v_issued - kAttnVStages; --j) {
          drained = mbar_wait(v_full(v_slot(j)), v_par(j), p.timeout_ns, nullptr);
        }
        if (!drained) attn_raise(p, abort_flag, kDevTimeoutDrain);
      }
      __syncwarp();
    } else if (warp == kAttnMmaWarp) {
      // ---- MMA issuer ----------------------------------------------------------
      if (lane == 0) {
        constexpr uint32_t idesc_s = idesc_bf16_f32(kAttnBQ, kAttnBKV, false, false);  // Q (K-major) x K^T (K-major)
        constexpr uint32_t idesc_o = idesc_bf16_f32(kAttnBQ, kAttnD, false, true);     // P (TMEM) x V (MN-major)
        // 16-wide K slices: K-major operands step 32 B inside a 64-wide atom
        // and 16 KiB between the two atoms; the MN-major V steps 16 keys =
        // 2 KiB inside a 64-key half and 16 KiB between halves; P in TMEM
        // steps 8 columns (16 bf16).
        auto kmajor = [](uint32_t tile, int k) {
          return smem_desc_sw128(tile + (uint32_t)((k >> 2) * 16384 + (k & 3) * 32), 16, 1024);
        };
        auto vdesc = [](uint32_t tile, int k) {
          return smem_desc_sw128(tile + (uint32_t)((k >> 2) * 16384 + (k & 3) * 2048), 8192, 1024);
        };
        auto issue_s = [&](int i, int j) {
          const uint32_t qa = sQ + (uint32_t)(i * Plan::kTileBytes);
          const uint32_t kt = sK + (uint32_t)(k_slot(j) * Plan::kTileBytes);
#pragma unroll
          for (int k = 0; k < kAttnD / kUmmaK; ++k) {
            umma_bf16(tmem_base + (uint32_t)(i * 128), kmajor(qa, k), kmajor(kt, k), idesc_s, k > 0 ? 1u : 0u);
          }
        };
        // Keys 64 h .. 64 h + 63 of P V (K slices 4 h .. 4 h + 3).
        auto issue_pv = [&](int i, int j, int h) {
          const uint32_t vt = sV + (uint32_t)(v_slot(j) * Plan::kTileBytes);
#pragma unroll
          for (int k = 4 * h; k < 4 * h + 4; ++k) {
            umma_bf16_ts(tmem_base + 256u + (uint32_t)(i * 128), tmem_base + (uint32_t)(i * 128 + k * 8),
                         vdesc(vt, k), idesc_o, (j > 0 || k > 0) ? 1u : 0u);
          }
        };
        auto wait_k = [&](int j) { return mbar_wait(k_full(k_slot(j)), k_par(j), p.timeout_ns, abort_flag); };
        bool ok = true;
        for (int i = 0; ok && i < n_q; ++i) ok = mbar_wait(q_full(i), 0u, p.timeout_ns, abort_flag);
        if (ok && n_max > 0) {
          ok = wait_k(0);
          if (ok) {
            tc_fence_after();
            for (int i = 0; i < n_q; ++i) {
              issue_s(i, 0);
              umma_commit(s_full(i));
            }
            umma_commit(k_empty(0));
          }
        }
        const int n_tiles[2] = {n0, n1};
        for (int j = 0; j < n_max && ok; ++j) {
          if (!mbar_wait(v_full(v_slot(j)), v_par(j), p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          bool k_ready = false;
#pragma unroll
          for (int i = 0; i < kAttnQTiles; ++i) {
            if (!ok || j >= n_tiles[i]) continue;
            // The first half of P V starts while the softmax still works on
            // the second half of the row.
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
            if (i == kAttnQTiles - 1 || j >= n_tiles[kAttnQTiles - 1]) umma_commit(v_empty(v_slot(j)));  // last user of V_j
            if (j + 1 < n_tiles[i]) {
              if (!k_ready) {
                if (!wait_k(j + 1)) {
                  ok = false;
                  continue;
                }
                k_ready = true;
                tc_fence_after();
              }
              issue_s(i, j + 1);
              umma_commit(s_full(i));
            } else {
              umma_commit(o_full(i));
            }
          }
          if (ok && j + 1 < n_max) umma_commit(k_empty(k_slot(j + 1)));
        }
        if (!ok) attn_raise(p, abort_flag, kDevTimeoutMma);
        umma_commit(drain);
        if (!mbar_wait(drain, 0u, p.timeout_ns, nullptr)) attn_raise(p, abort_flag, kDevTimeoutDrain);
      }
      __syncwarp();
    }
  } else {
    setmaxnreg_inc<kAttnRegsSoftmax>();
    // ---- softmax + epilogue (warps 0..3: tile 0, warps 4..7: tile 1) ----------
    const int tile = warp >> 2;
    const int qw = warp & 3;                // TMEM lane quarter this warp may access
    const int row = qw * 32 + (int)lane;     // query row in the tile
    const int qt = qt_of[tile];
    const int n_kv = tile == 0 ? n0 : n1;
    const int q_idx = qt * kAttnBQ + row;    // query position
    const uint32_t lane_off = (uint32_t)(qw * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + (uint32_t)(tile * 128);
    const uint32_t tO = tmem_base + lane_off + 256u + (uint32_t)(tile * 128);
    float m = -INFINITY;  // running max (exp2 domain) the stored P and O refer to
    float l = 0.0f;       // running sum of P
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
      const bool diag = p.causal && kv0 + kAttnBKV > qt * kAttnBQ;  // the tile crossing the diagonal
      // Only the diagonal tile and a tile past the sequence end need masks:
      // keys c >= lim are masked.
      const bool masked = diag || kv0 + kAttnBKV > p.seq_len;
      if (masked) {
        const int lim = min(p.seq_len - kv0, diag ? q_idx - kv0 + 1 : kAttnBKV);
#pragma unroll
        for (int c = 0; c < kAttnBKV; ++c) x[c] = c < lim ? x[c] : -INFINITY;
      }
      // Row max of the raw scores (the scale is positive): eight independent
      // chains of three-input maxima, so one thread's row is not one long
      // dependency chain.
      float mxs[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxs[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < kAttnBKV; c += 2) mxs[(c >> 1) & 7] = max3f(mxs[(c >> 1) & 7], x[c], x[c + 1]);
      const float mx = max3f(max3f(mxs[0], mxs[1], mxs[2]), max3f(mxs[3], mxs[4], mxs[5]), fmaxf(mxs[6], mxs[7]));
      const float m_new = fmaxf(m, mx * p.scale_log2);
      // Move the reference max only when the row max grew by more than 2^8
      // (or nothing was seen yet): P stays below 2^8, and O is rescaled rarely.
      const bool move = (m == -INFINITY) ? (m_new != -INFINITY) : (m_new > m + kAttnRescaleLog2);
      const float factor = (move && m != -INFINITY) ? fast_exp2(m - m_new) : 1.0f;
      const float m_next = move ? m_new : m;
      const float m_use = (m_next == -INFINITY) ? 0.0f : m_next;
      if (j > 0 && __any_sync(0xffffffffu, move && factor != 1.0f)) {
        // S_i(j) was issued after P_i(j-1) V(j-1), and its completion signal
        // covers that product: O is stable until this warpgroup's P is in.
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
      // P row -> TMEM over the first 64 columns of S (two bf16 per column),
      // in two halves of 64 keys, each published as soon as it is stored.
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t pw[32];
        l += masked ? row_exp<64, false>(x + 64 * h, p.scale_log2, m_use, pw)
                    : row_exp<64, true>(x + 64 * h, p.scale_log2, m_use, pw);
        tmem_st_32x32b_x32(tS + (uint32_t)(32 * h), pw);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(tile, h));
      }
    }
    if (!ok) {
      if (lane == 0) attn_raise(p, abort_flag, kDevTimeoutEpilogue);
    } else if (n_kv > 0) {
      // O / l -> bf16 -> TMA store, through this warp's 8 KiB of the tile's
      // Q buffer (idle once the last product is done): two [32 rows][64 d]
      // swizzled chunks.
      const bool last = mbar_wait(o_full(tile), 0u, p.timeout_ns, abort_flag);
      if (__all_sync(0xffffffffu, last)) {
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
      } else if (lane == 0) {
        attn_raise(p, abort_flag, kDevTimeoutEpilogue);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kAttnMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
#endif  // B200_NO_SM100A_FEATURES
}

}  // namespace b200
