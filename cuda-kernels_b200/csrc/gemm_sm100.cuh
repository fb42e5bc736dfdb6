// Persistent, warp-specialised BF16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M,N] (bf16, row-major) = A[M,K] (bf16, row-major) x B, fp32 accumulate,
//   B stored either [N,K] row-major ("K-major", the reference's layout:
//   bf16_matmul/README.md:7, bf16_matmul/matmul_v8_tuned.cu:214) or [K,N]
//   row-major ("MN-major").
//
// This replaces the reference's one-CTA-per-tile mma.sync kernel
// (bf16_matmul/matmul_v8_tuned.cu:30-179).  The design is Blackwell-first:
//
//   warp 0      TMA producer: one lane streams 128B-swizzled A/B K-blocks into
//               a STAGES-deep shared-memory ring (full/empty mbarriers).
//   warp 1      MMA issuer: allocates TMEM, one lane issues tcgen05.mma
//               (M=128, N=BN, K=16) into a double-buffered fp32 accumulator
//               in TMEM and releases ring stages with tcgen05.commit.
//   warps 2..5  epilogue: tcgen05.ld TMEM -> registers, round to bf16 (RN),
//               stage through 128B-swizzled shared memory, TMA-store.  Runs
//               on accumulator buffer b while the MMA warp fills buffer b^1.
//
// Tiles are visited persistently (grid <= #SMs) in grouped order along M so
// that the tiles in flight at any moment share A row panels and B column
// panels in L2.  Out-of-range rows/columns/K are handled by TMA: loads fill
// zeros, stores are clipped, so any M, N, K >= 1 works (row pitches must be
// multiples of 8 elements for TMA).
#pragma once

#include <cuda.h>  // CUtensorMap (type only; no driver symbols are linked)
#include <cuda_bf16.h>
#include <cstdint>

#include "ptx_sm100.cuh"

namespace b200 {

constexpr int kBM = 128;          // UMMA M (one CTA)
constexpr int kBK = 64;           // one 128-byte swizzle row of bf16 per K-block
constexpr int kUmmaK = 16;        // K per tcgen05.mma kind::f16
constexpr int kNumThreads = 192;  // 6 warps
constexpr int kEpiWarps = 4;
constexpr int kAccBufs = 2;
constexpr int kTmemCols = 512;
constexpr int kEpiCols = 64;             // columns per epilogue chunk (one 128B swizzle row of bf16)
constexpr int kEpiRowsPerWarp = 32;
constexpr int kEpiBufBytes = kEpiRowsPerWarp * kEpiCols * 2;  // 4 KiB

// Optional fused epilogue (b200_gemm_bf16_ex): D = alpha * acc + bias[n] +
// beta * C_in[m, n], rounded to bf16 or kept in fp32.  The operations are
// done one at a time in fp32, in that order, without contraction into FMAs,
// so a CPU restatement reproduces them exactly from the same fp32 acc.
// `active` == 0 is the plain GEMM (D = bf16(acc)) with no extra work.
struct EpilogueParams {
  const __nv_bfloat16* c_in;  // [M, N] row-major, leading dimension ldc_in; read only when beta != 0
  const __nv_bfloat16* bias;  // [N] or nullptr
  int64_t ldc_in;
  float alpha, beta;
  uint32_t out_f32;  // element type of D: 0 bf16, 1 fp32
  uint32_t active;
};

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }

// 32 consecutive columns n0 .. n0+31 of row m, held by one thread as fp32
// bit patterns: apply the epilogue in place, 8 columns (one 16-byte load of
// bias and of C_in) at a time.  Columns >= N and rows >= M read nothing
// (their results are never stored).  C_in is read with plain loads: it may be
// D itself, whose other elements TMA stores are writing meanwhile.
__device__ __forceinline__ void epilogue_row32(uint32_t (&v)[32], const EpilogueParams& e, int m, int n0, int M,
                                               int N) {
  const bool use_c = e.beta != 0.0f && m < M;
  const unsigned short* bias = reinterpret_cast<const unsigned short*>(e.bias);
  const unsigned short* crow =
      use_c ? reinterpret_cast<const unsigned short*>(e.c_in) + (size_t)m * (size_t)e.ldc_in : nullptr;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int n = n0 + 8 * g;
    uint32_t bw[4] = {0u, 0u, 0u, 0u}, cw[4] = {0u, 0u, 0u, 0u};
    if (n + 8 <= N) {
      if (bias != nullptr) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(bias + n));
        bw[0] = w.x; bw[1] = w.y; bw[2] = w.z; bw[3] = w.w;
      }
      if (use_c) {
        const uint4 w = ld_global_v4_u32(crow + n);
        cw[0] = w.x; cw[1] = w.y; cw[2] = w.z; cw[3] = w.w;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (n + i < N) {
          const uint32_t sh = (i & 1) * 16u;
          if (bias != nullptr) bw[i >> 1] |= (uint32_t)__ldg(bias + n + i) << sh;
          if (use_c) cw[i >> 1] |= ld_global_u16(crow + n + i) << sh;
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b16 = (bw[i >> 1] >> ((i & 1) * 16u)) & 0xffffu;
      const uint32_t c16 = (cw[i >> 1] >> ((i & 1) * 16u)) & 0xffffu;
      float x = __fmul_rn(e.alpha, __uint_as_float(v[8 * g + i]));
      x = __fadd_rn(x, bf16_bits_to_f32(b16));
      x = __fadd_rn(x, __fmul_rn(e.beta, bf16_bits_to_f32(c16)));
      v[8 * g + i] = __float_as_uint(x);
    }
  }
}

// Stage one thread's 64 columns (lo = columns 0..31, hi = 32..63) of a warp's
// 32-row block into 128B-swizzled shared memory for the TMA store of D.
// bf16 D: one 4 KiB buffer [32 rows][64 cols].  fp32 D: two 4 KiB buffers
// [32 rows][32 cols] (lo into buf0, hi into buf1).
__device__ __forceinline__ void stage_row64(const uint32_t (&lo)[32], const uint32_t (&hi)[32], bool f32,
                                            uint32_t buf0, uint32_t buf1, uint32_t lane) {
  if (!f32) {
    const uint32_t row_addr = buf0 + lane * 128u;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t* src = (j < 4) ? &lo[j * 8] : &hi[(j - 4) * 8];
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        __nv_bfloat162 h = __floats2bfloat162_rn(__uint_as_float(src[2 * e]), __uint_as_float(src[2 * e + 1]));
        w[e] = *reinterpret_cast<uint32_t*>(&h);
      }
      const uint32_t dst = row_addr + (((uint32_t)j ^ (lane & 7u)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3])
                   : "memory");
    }
  } else {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t* src = half == 0 ? lo : hi;
      const uint32_t row_addr = (half == 0 ? buf0 : buf1) + lane * 128u;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t dst = row_addr + (((uint32_t)j ^ (lane & 7u)) << 4);
        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst), "r"(src[4 * j]), "r"(src[4 * j + 1]),
                     "r"(src[4 * j + 2]), "r"(src[4 * j + 3])
                     : "memory");
      }
    }
  }
}

// Epilogue helper: while the tile's MMAs still run, pull this thread's row
// segment of C_in, columns [n0, n0 + cols), into L2 (clipped to N; the size
// is rounded up to 8 elements, which stays inside the row since ldc_in is a
// multiple of 8 and >= N).
__device__ __forceinline__ void epilogue_prefetch_row(const EpilogueParams& e, int m, int n0, int cols, int M,
                                                      int N) {
  if (e.beta == 0.0f || m >= M || n0 >= N) return;
  const int n = min(cols, N - n0);
  prefetch_l2_bulk(e.c_in + (size_t)m * (size_t)e.ldc_in + n0, (uint32_t)((n + 7) & ~7) * 2u);
}

struct GemmParams {
  int32_t M, N, K;
  int32_t num_m_blk, num_n_blk, num_k_blk;
  int32_t num_tiles;
  int32_t group_m;       // tiles are rasterised in groups of `group_m` M-blocks
  uint32_t b_mn_major;   // 0: B is [N,K] (K contiguous); 1: B is [K,N] (N contiguous)
  // Split-K tail (pair kernel only).  Work items [0, sk_first) are whole tiles
  // 0 .. sk_first-1.  Each tile from sk_first on is split into sk_parts
  // ranges of sk_kpp K-blocks, one work item per range; parts 0..sk_parts-2
  // write fp32 partial tiles to `workspace` and publish `epoch` in `flags`;
  // the last part adds the partials (in part order) and stores C.  Without a
  // split: sk_first = num_work = num_tiles.
  int32_t sk_first, sk_parts, sk_kpp, num_work;
  uint64_t epoch;        // per-launch tag: random per-process high half, launch counter low half
  uint64_t timeout_ns;   // limit for every mbarrier wait
  uint32_t* status;      // device status word (DeviceStatus bits), OR-ed on failure
  float* workspace;      // [split tiles][sk_parts-1][2 CTAs][BN/4][128][4] fp32
  uint64_t* flags;       // [split tiles][sk_parts-1][2 CTAs]
  EpilogueParams epi;
  int32_t num_out;       // output tensor maps each C tile is stored to (1, or one per rank when gathering)
  // Exchange hooks (pair kernel, b200_bcast_gemm): B is a receive slot that
  // other GPUs fill.  Every producer waits until each dep flag has reached
  // dep_value before its first load; once all of the grid's loads have
  // landed, the last CTA pair writes rel_value into every rel flag (the
  // writers' "slot free" flags, in their memory) and resets rel_counter.
  const uint32_t* dep_flags[8];
  uint32_t* rel_flags[8];
  uint32_t* rel_counter;
  int32_t n_dep, n_rel;
  uint32_t dep_value, rel_value;
};

// Exchange hooks of GemmParams: producer side.  Returns false when a flag
// did not arrive in time.
__device__ __forceinline__ bool wait_deps(const GemmParams& p) {
  for (int i = 0; i < p.n_dep; ++i) {
    if (!wait_flag_reached(p.dep_flags[i], p.dep_value, p.timeout_ns)) return false;
  }
  fence_proxy_async_global();  // the flags' acquire comes before this thread's TMA reads of B
  return true;
}
// Called once per CTA pair (its leader's producer) after every load of the
// pair has landed, also on an error path (the writers must not wait for a
// release that never comes).  The last pair to finish releases the slot.
__device__ __forceinline__ void release_slot(const GemmParams& p, int num_pairs) {
  if (p.rel_counter == nullptr) return;
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(p.rel_counter) : "memory");
  if (old + 1u == (uint32_t)num_pairs) {
    for (int i = 0; i < p.n_rel; ++i) st_release_sys_u32(p.rel_flags[i], p.rel_value);
    asm volatile("st.relaxed.gpu.global.u32 [%0], 0;" ::"l"(p.rel_counter) : "memory");
  }
}

// Output tensor maps of the gathering GEMM (b200_gemm_bf16_allgather): the
// rows this rank computes, in every rank's gathered C, each mapped in this
// process (peer buffers through CUDA IPC).
constexpr int kMaxOutMaps = 8;
struct OutMaps {
  CUtensorMap m[kMaxOutMaps];
};

template <int BN, int STAGES>
struct SmemPlan {
  static constexpr int kABytes = kBM * kBK * 2;  // 16 KiB
  static constexpr int kBBytes = BN * kBK * 2;   // 32 KiB for BN=256
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kOffA = 0;
  static constexpr int kOffB = kOffA + STAGES * kABytes;
  static constexpr int kOffC = kOffB + STAGES * kBBytes;
  static constexpr int kOffBar = kOffC + kEpiWarps * 2 * kEpiBufBytes;
  // barriers: full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * STAGES + 2 * kAccBufs + 1;
  static constexpr int kOffTmemHolder = kOffBar + kNumBars * 8;
  static constexpr int kOffAbort = kOffTmemHolder + 4;
  static constexpr int kBytes = kOffAbort + 4;
  static constexpr int kAllocBytes = kBytes + 1024;  // slack for 1024-byte alignment
  static_assert(kAllocBytes <= 232448, "shared memory plan exceeds 227 KiB");
};

__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& mb, int& nb) {
  const int tiles_per_group = p.group_m * p.num_n_blk;
  const int g = t / tiles_per_group;
  const int first_m = g * p.group_m;
  const int gm = min(p.num_m_blk - first_m, p.group_m);
  const int r = t - g * tiles_per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

struct WorkItem {
  int mb, nb;    // tile coordinates
  int part;      // -1: whole K range; otherwise the split-K part index
  int kb0, kb1;  // K-block range [kb0, kb1)
  int split;     // index of the split tile (w.r.t. sk_first), or -1
};

__device__ __forceinline__ WorkItem work_item(int w, const GemmParams& p) {
  WorkItem r;
  if (w < p.sk_first) {
    tile_coords(w, p, r.mb, r.nb);
    r.part = -1;
    r.kb0 = 0;
    r.kb1 = p.num_k_blk;
    r.split = -1;
  } else {
    const int u = w - p.sk_first;
    r.split = u / p.sk_parts;
    r.part = u - r.split * p.sk_parts;
    tile_coords(p.sk_first + r.split, p, r.mb, r.nb);
    r.kb0 = r.part * p.sk_kpp;
    r.kb1 = min(r.kb0 + p.sk_kpp, p.num_k_blk);
  }
  return r;
}

__device__ __forceinline__ void raise_status(const GemmParams& p, volatile uint32_t* abort_flag, uint32_t code) {
  *abort_flag = 1u;
  if (p.status != nullptr) atomicOr(p.status, code);
}

template <int BN, int STAGES, bool B_MN, bool EPI = false>
__global__ void __launch_bounds__(kNumThreads, 1)
    gemm_bf16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmC, const GemmParams p) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && p.status != nullptr) atomicOr(p.status, (uint32_t)kDevWrongArch);
#else
  using Plan = SmemPlan<BN, STAGES>;
  static_assert(BN % kEpiCols == 0 && BN >= 64 && BN <= 256, "BN must be 64..256 in steps of 64");
  static_assert(kAccBufs * BN <= kTmemCols, "accumulators must fit in TMEM");

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
  auto acce_bar = [&](int b) { return bar0 + 8u * (2 * STAGES + kAccBufs + b); };
  const uint32_t drain_bar = bar0 + 8u * (2 * STAGES + 2 * kAccBufs);
  volatile uint32_t* tmem_holder = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffTmemHolder);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(base_ptr + Plan::kOffAbort);

  const int warp = threadIdx.x >> 5;
  const uint32_t lane = threadIdx.x & 31u;

  // ---- set-up -------------------------------------------------------------
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), kEpiWarps);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0u;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    tma_prefetch_desc(&tmC);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_holder)), kTmemCols);
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
    // ---- TMA producer -------------------------------------------------------
    if (lane == 0) {
      // Operand tiles are re-read by the other tiles of their row / column
      // block: keep them in L2 ahead of the output stream (B200: 2-3 % at
      // 4096^3 and 8192^3, from fewer DRAM trips under the power cap).
      const uint64_t pol = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;  // total K-blocks loaded by this CTA
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, p, mb, nb);
        for (int kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1u, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, Plan::kStageBytes);
          tma_load_2d(sA + stage * Plan::kABytes, &tmA, fb, kb * kBK, mb * kBM, pol);
          const uint32_t dstB = sB + stage * Plan::kBBytes;
          if constexpr (!B_MN) {
            tma_load_2d(dstB, &tmB, fb, kb * kBK, nb * BN, pol);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) {
              tma_load_2d(dstB + j * (64 * kBK * 2), &tmB, fb, nb * BN + 64 * j, kb * kBK, pol);
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
      // Drain: the most recent load into every stage must have landed before
      // this CTA may exit (its destination is this CTA's shared memory).
      const uint32_t nst = issued < (uint32_t)STAGES ? issued : (uint32_t)STAGES;
      for (uint32_t i = 0; i < nst; ++i) {
        const uint32_t it = issued - 1u - i;  // iteration index of a recent load
        const uint32_t s = it % STAGES;
        const uint32_t par = (it / STAGES) & 1u;
        if (!mbar_wait(full_bar(s), par, p.timeout_ns, nullptr)) {
          raise_status(p, abort_flag, kDevTimeoutDrain);
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issuer ---------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN, false, B_MN);
      // Stage-0 descriptors (layouts as in gemm_sm100_pair.cuh); stages and
      // K slices only advance the start-address field.
      const uint64_t a_desc0 = smem_desc_sw128(sA, 16, 1024);
      const uint64_t b_desc0 = B_MN ? smem_desc_sw128(sB, 64 * kBK * 2, 1024) : smem_desc_sw128(sB, 16, 1024);
      constexpr uint32_t kBStep = B_MN ? (2048 >> 4) : (32 >> 4);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(acce_bar(acc), acc_phase ^ 1u, p.timeout_ns, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < p.num_k_blk; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, p.timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = a_desc0 + (uint64_t)((stage * Plan::kABytes) >> 4);
          const uint64_t bd = b_desc0 + (uint64_t)((stage * Plan::kBBytes) >> 4);
#pragma unroll
          for (int k = 0; k < kBK / kUmmaK; ++k) {
            umma_bf16(d_tmem, ad + 2u * k, bd + kBStep * k, idesc, (kb | k) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));  // stage is free once these MMAs have read it
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(accf_bar(acc));  // accumulator ready for the epilogue
        if (++acc == kAccBufs) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      if (!ok) raise_status(p, abort_flag, kDevTimeoutMma);
      // Drain: every MMA issued by this thread must finish before TMEM is freed.
      umma_commit(drain_bar);
      if (!mbar_wait(drain_bar, 0u, p.timeout_ns, nullptr)) raise_status(p, abort_flag, kDevTimeoutDrain);
    }
    __syncwarp();
  } else {
    // ---- epilogue (warps 2..5) ----------------------------------------------
    const int q = warp & 3;            // TMEM lane quarter this warp may access
    const int slot = warp - 2;         // private staging buffers
    const uint32_t tmem_lane = (uint32_t)(q * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    int sbuf = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x) {
      int mb, nb;
      tile_coords(t, p, mb, nb);
      if constexpr (EPI) epilogue_prefetch_row(p.epi, mb * kBM + q * kEpiRowsPerWarp + (int)lane, nb * BN, BN, p.M, p.N);
      const bool got = mbar_wait(accf_bar(acc), acc_phase, p.timeout_ns, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        if (lane == 0) raise_status(p, abort_flag, kDevTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      const uint32_t t_row = tmem_base + tmem_lane + (uint32_t)(acc * BN);
#pragma unroll 1
      for (int c = 0; c < BN / kEpiCols; ++c) {
        uint32_t r0[32], r1[32];
        tmem_ld_32x32b_x32(t_row + c * kEpiCols, r0);
        tmem_ld_32x32b_x32(t_row + c * kEpiCols + 32, r1);
        tmem_ld_wait_regs(r0);
        tmem_ld_wait_regs(r1);
        if (c == BN / kEpiCols - 1) {
          // All TMEM reads of this accumulator are complete: hand it back.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acce_bar(acc));
        }
        const int n0 = nb * BN + c * kEpiCols;
        const int m0 = mb * kBM + q * kEpiRowsPerWarp;
        if constexpr (EPI) {
          if (p.epi.active) {
            epilogue_row32(r0, p.epi, m0 + (int)lane, n0, p.M, p.N);
            epilogue_row32(r1, p.epi, m0 + (int)lane, n0 + 32, p.M, p.N);
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
          tma_store_2d(&tmC, buf0, n0, m0);
          if (f32) tma_store_2d(&tmC, buf1, n0 + 32, m0);
          bulk_commit_group();
        }
        sbuf ^= 1;
      }
      if (++acc == kAccBufs) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
    if (lane == 0) bulk_wait_group_read<0>();  // smem reads done; the global writes complete with the grid
    __syncwarp();
  }

  // ---- teardown -------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
#endif  // B200_NO_SM100A_FEATURES
}

}  // namespace b200
