// Host side of the C ABI declared in include/b200_gemm.h.
//
// Responsibilities: argument checking (the reference only host-asserts tile
// multiples, bf16_matmul/matmul_v8_tuned.cu:238), TMA descriptor encoding
// (the reference links -lcuda and calls cuTensorMapEncodeTiled directly,
// matmul_v8_tuned.cu:181-210; here the driver entry point is fetched through
// the runtime so nothing links against libcuda), per-device one-time set-up
// (SM count, shared-memory opt-in, status word), and the persistent launch.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdint>
#include <random>
#include <cstring>
#include <mutex>

#include "b200_gemm.h"  // include/ (pass -I <repo>/include)
#include "gemm_sm100.cuh"
#include "gemm_sm100_pair.cuh"
#include "gemm_sm100_skinny.cuh"
#include "split_f32.cuh"
#include "attn_sm100.cuh"
#include "attn_sm100_pair.cuh"
#include "peer_bcast.h"

namespace {

// Device status word.  Kernels OR DeviceStatus bits into it when a bounded
// wait gives up; b200_gemm_status() reads and clears it.
__device__ uint32_t g_b200_status;

constexpr int kMaxDevices = 64;
constexpr uint64_t kDefaultTimeoutNs = 4000000000ull;  // 4 s: far above any legitimate wait

// Kernel configurations shipped by the library.
//   single: one CTA per 128 x 256 tile, 4-stage ring   (M <= 128)
//   pair:   a CTA pair per 256 x 256 tile, 6-stage ring (everything else)
constexpr int kBN = 256;
constexpr int kStages = 4;
// Small problems (a 256 x 256 pair tiling would leave most SMs idle): one CTA
// per 128 x 64 tile, so up to one tile per SM.
constexpr int kSmallBN = 64;
constexpr int kSmallStages = 8;
constexpr int kPairBN = 256;
constexpr int kPairStages = 6;
// Wide pair tiles (256 x 512): each CTA reuses its A rows for 512 output
// columns, 25 % fewer operand bytes per FLOP than 256 x 256, and 8 MMAs per
// ring stage.  Used when there is at least one wide tile per CTA pair.
constexpr int kPairWideBN = 512;
constexpr int kPairWideStages = 4;
constexpr int kGroupM = 16;

// Skinny (M <= 128) configurations: UMMA N = MPAD, ring depth per MPAD.
// (Measured on B200: rings of 4-5 stages, small enough for two CTAs per SM
// so that the next launch's CTAs could prefetch its weights while this one
// runs, were 10-20 % slower in back-to-back launches.)
template <int MPAD>
struct SkinnyCfg;
template <>
struct SkinnyCfg<16> { static constexpr int kStages = 10; };
template <>
struct SkinnyCfg<32> { static constexpr int kStages = 9; };
template <>
struct SkinnyCfg<64> { static constexpr int kStages = 8; };
template <>
struct SkinnyCfg<128> { static constexpr int kStages = 6; };
constexpr int kMaxClusterSplits = 8;  // portable cluster size limit

// Kernel selection override (b200_gemm_set_kernel): process-wide.
enum ForceKernel { kForceAuto = 0, kForceSingle = 1, kForcePair = 2, kForceSkinny = 3 };
std::atomic<int> g_force_kernel{kForceAuto};
std::atomic<int> g_attn_kernel{B200_ATTN_KERNEL_AUTO};

struct DeviceState {
  std::once_flag once;
  int init_rc = B200_OK;
  int sm_count = 0;
  int max_pairs = 0;  // co-resident 2-CTA clusters of the pair kernel
  uint32_t* status_ptr = nullptr;
  uint64_t timeout_ns = kDefaultTimeoutNs;
  std::atomic<uint32_t> epoch{0};  // split-K hand-off counter, one step per launch
  // The attention kernel moves registers between warpgroups (setmaxnreg); its
  // shares add up to exactly the pool of a launch at kAttnRegsLaunch
  // registers per thread, so it only runs when the binary has that count.
  bool attn_regs_ok = false;
  bool attn_pair_regs_ok = false;  // the same for the CTA-pair attention kernel
  // Same for the eight-epilogue-warp wide pair kernel (kWide8Regs*); when the
  // binary has another count, the four-warp wide kernel is used instead.
  bool wide8_regs_ok = false;
};

// Split-K plan for the pair kernel's last, partial wave of tiles (see
// GemmParams): the `rem` tiles left after the full waves are each split into
// `parts` K ranges so that rem x parts work items fill the pairs again.
struct SplitPlan {
  int32_t first, parts, kpp, work;
  size_t partial_bytes, flag_bytes;
  size_t bytes() const { return partial_bytes + flag_bytes; }
};
constexpr size_t kWsAlign = 256;

uint32_t process_salt() {
  static const uint32_t salt = [] {
    std::random_device rd;
    uint32_t v = rd() ^ (uint32_t)std::chrono::steady_clock::now().time_since_epoch().count();
    return v == 0 ? 0x9e3779b9u : v;
  }();
  return salt;
}

SplitPlan plan_split(int64_t tiles, int32_t num_k_blk, int max_pairs, int bn) {
  SplitPlan sp{(int32_t)tiles, 1, num_k_blk, (int32_t)tiles, 0, 0};
  if (max_pairs <= 0) return sp;
  const int64_t rem = tiles % max_pairs;
  if (rem == 0) return sp;
  int64_t parts = max_pairs / rem;
  if (parts > 8) parts = 8;
  // Each part must keep enough K to amortise the partial hand-off (a 256 KB
  // fp32 tile written and read back per part); measured on B200: 4 K-blocks
  // per part made 1024^3 1.7x slower, 32 per part made 4096^3 faster.
  constexpr int32_t kMinKbPerPart = 16;
  if (parts > num_k_blk / kMinKbPerPart) parts = num_k_blk / kMinKbPerPart;
  if (parts < 2) return sp;
  const int32_t kpp = (int32_t)((num_k_blk + parts - 1) / parts);
  parts = (num_k_blk + kpp - 1) / kpp;
  if (parts < 2) return sp;
  sp.first = (int32_t)(tiles - rem);
  sp.parts = (int32_t)parts;
  sp.kpp = kpp;
  sp.work = (int32_t)(sp.first + rem * parts);
  const size_t slots = (size_t)rem * (size_t)(parts - 1) * 2;  // 2 CTAs per pair
  sp.partial_bytes = (slots * (size_t)b200::kBM * (size_t)bn * sizeof(float) + kWsAlign - 1) / kWsAlign * kWsAlign;
  sp.flag_bytes = (slots * sizeof(uint64_t) + kWsAlign - 1) / kWsAlign * kWsAlign;
  return sp;
}

DeviceState g_dev[kMaxDevices];

std::once_flag g_encode_once;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

void load_encode_fn() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess) {
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
}

template <int MPAD>
int set_skinny_attrs() {
  constexpr int st = SkinnyCfg<MPAD>::kStages;
  constexpr int smem = b200::SkinnySmemPlan<MPAD, st>::kAllocBytes;
  constexpr int smem_epi = b200::SkinnySmemPlan<MPAD, st>::kAllocBytesEpi;
  const void* kernels[4] = {(const void*)b200::gemm_bf16_skinny_kernel<MPAD, st, false, false>,
                            (const void*)b200::gemm_bf16_skinny_kernel<MPAD, st, true, false>,
                            (const void*)b200::gemm_bf16_skinny_kernel<MPAD, st, false, true>,
                            (const void*)b200::gemm_bf16_skinny_kernel<MPAD, st, true, true>};
  for (int i = 0; i < 4; ++i) {
    if (cudaFuncSetAttribute(kernels[i], cudaFuncAttributeMaxDynamicSharedMemorySize, i < 2 ? smem : smem_epi) !=
        cudaSuccess)
      return B200_ERR_CUDA;
  }
  return B200_OK;
}

int init_device(int dev, DeviceState& st) {
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return B200_ERR_CUDA;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return B200_ERR_CUDA;
  if (major != 10 || minor != 0) return B200_ERR_UNSUPPORTED_DEVICE;
  if (cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return B200_ERR_CUDA;
  if (cudaGetSymbolAddress(reinterpret_cast<void**>(&st.status_ptr), g_b200_status) != cudaSuccess)
    return B200_ERR_CUDA;
  constexpr int single_smem = b200::SmemPlan<kBN, kStages>::kAllocBytes;
  constexpr int small_smem = b200::SmemPlan<kSmallBN, kSmallStages>::kAllocBytes;
  constexpr int pair_smem = b200::PairSmemPlan<kPairBN, kPairStages>::kAllocBytes;
  constexpr int wide_smem = b200::PairSmemPlan<kPairWideBN, kPairWideStages>::kAllocBytes;
  struct KernelSmem {
    const void* fn;
    int smem;
  };
  const KernelSmem kernels[] = {
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kBN, kStages, false, false>, single_smem},
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kBN, kStages, true, false>, single_smem},
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kBN, kStages, false, true>, single_smem},
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kBN, kStages, true, true>, single_smem},
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, false, false>, small_smem},
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, true, false>, small_smem},
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, false, true>, small_smem},
      {(const void*)b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, true, true>, small_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, false, false>, pair_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, true, false>, pair_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, false, true>, pair_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, true, true>, pair_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, false, false>, wide_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, true, false>, wide_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, false, true>, wide_smem},
      {(const void*)b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, true, true>, wide_smem},
      {(const void*)b200::gemm_bf16_pair_gather_kernel<false>, pair_smem},
      {(const void*)b200::gemm_bf16_pair_gather_kernel<true>, pair_smem},
  };
  for (const KernelSmem& k : kernels) {
    if (cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize, k.smem) != cudaSuccess)
      return B200_ERR_CUDA;
  }
  if (cudaFuncSetAttribute(b200::flash_attn_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           b200::AttnSmemPlan::kAllocBytes) != cudaSuccess)
    return B200_ERR_CUDA;
  {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, b200::flash_attn_fwd_kernel) != cudaSuccess) return B200_ERR_CUDA;
    st.attn_regs_ok = fa.numRegs == (int)b200::kAttnRegsLaunch;
  }
  if (cudaFuncSetAttribute(b200::flash_attn_fwd_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           b200::AttnPairSmemPlan::kAllocBytes) != cudaSuccess)
    return B200_ERR_CUDA;
  {
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, b200::flash_attn_fwd_pair_kernel) != cudaSuccess) return B200_ERR_CUDA;
    st.attn_pair_regs_ok = fa.numRegs == (int)b200::kAttnRegsLaunch;
  }
  {
    st.wide8_regs_ok = true;
    const void* w8[2] = {(const void*)b200::gemm_bf16_pair_wide8_kernel<false>,
                         (const void*)b200::gemm_bf16_pair_wide8_kernel<true>};
    for (const void* k : w8) {
      if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, wide_smem) != cudaSuccess)
        return B200_ERR_CUDA;
      cudaFuncAttributes fa{};
      if (cudaFuncGetAttributes(&fa, k) != cudaSuccess) return B200_ERR_CUDA;
      if (fa.numRegs != (int)b200::kWide8RegsLaunch) st.wide8_regs_ok = false;
    }
  }
  if (set_skinny_attrs<16>() != B200_OK || set_skinny_attrs<32>() != B200_OK || set_skinny_attrs<64>() != B200_OK ||
      set_skinny_attrs<128>() != B200_OK)
    return B200_ERR_CUDA;
  auto pkern = b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, false>;
  {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * (st.sm_count / 2), 1, 1);
    cfg.blockDim = dim3(b200::kNumThreads, 1, 1);
    cfg.dynamicSmemBytes = pair_smem;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, pkern, &cfg) != cudaSuccess || clusters <= 0) return B200_ERR_CUDA;
    st.max_pairs = clusters;
  }
  std::call_once(g_encode_once, load_encode_fn);
  if (g_encode == nullptr) return B200_ERR_CUDA;
  return B200_OK;
}

int current_device_state(DeviceState** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return B200_ERR_UNSUPPORTED_DEVICE;
  DeviceState& st = g_dev[dev];
  std::call_once(st.once, [&] { st.init_rc = init_device(dev, st); });
  if (st.init_rc != B200_OK) return st.init_rc;
  *out = &st;
  return B200_OK;
}

// Tensor maps are pure host-side descriptors; repeated calls on the same
// buffers (the common case for weights and reused activations) skip the
// encode.  One small cache per host thread: no locking on the launch path.
struct TmapKey {
  const void* ptr;
  uint64_t inner, outer, pitch;
  uint32_t box_inner, box_outer;
  uint32_t flags;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && inner == o.inner && outer == o.outer && pitch == o.pitch && box_inner == o.box_inner &&
           box_outer == o.box_outer && flags == o.flags;
  }
};
constexpr int kTmapCacheSize = 32;
struct TmapCache {
  TmapKey key[kTmapCacheSize];
  CUtensorMap map[kTmapCacheSize];
  bool used[kTmapCacheSize] = {};
  int next = 0;
};
thread_local TmapCache t_tmap_cache;

int encode_2d_uncached(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t pitch_elems,
                       uint32_t box_inner, uint32_t box_outer, bool is_load, bool swizzle, bool f32) {
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_elems * (f32 ? 4 : 2)};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                        const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        is_load ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_NONE,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TENSOR_MAP;
}

// 2-D tensor map (bf16, or fp32 with f32 = true): `inner` contiguous
// elements per row, `outer` rows, `pitch_elems` elements between rows, box
// {box_inner, box_outer}, 128B swizzle unless `swizzle` is false.
int encode_2d(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t outer, uint64_t pitch_elems,
              uint32_t box_inner, uint32_t box_outer, bool is_load, bool swizzle = true, bool f32 = false) {
  TmapCache& c = t_tmap_cache;
  const TmapKey k{ptr,       inner,     outer,
                  pitch_elems, box_inner, box_outer,
                  (is_load ? 1u : 0u) | (swizzle ? 2u : 0u) | (f32 ? 4u : 0u)};
  for (int i = 0; i < kTmapCacheSize; ++i) {
    if (c.used[i] && c.key[i] == k) {
      *map = c.map[i];
      return B200_OK;
    }
  }
  const int rc = encode_2d_uncached(map, ptr, inner, outer, pitch_elems, box_inner, box_outer, is_load, swizzle, f32);
  if (rc == B200_OK) {
    const int i = c.next;
    c.next = (c.next + 1) % kTmapCacheSize;
    c.key[i] = k;
    c.map[i] = *map;
    c.used[i] = true;
  }
  return rc;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Swap-AB split-K launch for M <= 128 (see gemm_sm100_skinny.cuh).
template <int MPAD>
int launch_skinny(const DeviceState& st, const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                  int64_t lda, int64_t ldb, int64_t ldc, int b_layout, const b200::EpilogueParams& epi,
                  cudaStream_t stream) {
  constexpr int stages = SkinnyCfg<MPAD>::kStages;
  using Plan = b200::SkinnySmemPlan<MPAD, stages>;
  CUtensorMap tmB, tmA, tmC;
  int rc;
  if (b_layout == B200_B_NK) {
    rc = encode_2d(&tmB, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, b200::kBK, b200::kSkinnyBN, true);
  } else {
    rc = encode_2d(&tmB, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, b200::kBK, true);
  }
  if (rc != B200_OK) return rc;
  if ((rc = encode_2d(&tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, b200::kBK, MPAD, true)) != B200_OK) return rc;

  b200::SkinnyParams p{};
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.K = (int32_t)K;
  p.num_k_blk = (int32_t)((K + b200::kBK - 1) / b200::kBK);
  const int64_t n_tiles = (N + b200::kSkinnyBN - 1) / b200::kSkinnyBN;
  if (n_tiles > 65535) return B200_ERR_TOO_LARGE;  // grid.y limit
  // Split K so that tiles x splits CTAs cover the SMs once; the split count
  // is a power of two (each CTA of a cluster owns 128/S rows of the
  // reduction), at most 8 (portable cluster size) and at most what the
  // reduction scratch allows.  A split may end up with no K-blocks (it then
  // contributes zeros).
  int64_t cap = st.sm_count / n_tiles;
  if (cap > kMaxClusterSplits) cap = kMaxClusterSplits;
  if (cap > Plan::max_splits()) cap = Plan::max_splits();
  if (cap > p.num_k_blk) cap = p.num_k_blk;
  int64_t splits = 1;
  while (splits * 2 <= cap) splits *= 2;
  p.kb_per_split = (int32_t)((p.num_k_blk + splits - 1) / splits);
  p.splits = (int32_t)splits;
  // C store box: each warp stores [MPAD x 32] without a split; with S splits
  // each CTA stores its owned rows as one [MPAD x 128/S] block.
  const uint32_t box_n = (uint32_t)(splits == 1 ? 32 : b200::kSkinnyBN / splits);
  if ((rc = encode_2d(&tmC, C, (uint64_t)N, (uint64_t)M, (uint64_t)ldc, box_n, MPAD, false, false,
                      epi.out_f32 != 0)) != B200_OK)
    return rc;
  p.timeout_ns = st.timeout_ns;
  p.status = st.status_ptr;
  p.epi = epi;

  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)splits, (unsigned)n_tiles, 1);
  cfg.blockDim = dim3(b200::kNumThreads, 1, 1);
  // The fused-epilogue variants only when needed: the plain ones carry no
  // epilogue code at all.
  const bool fused = epi.active || epi.out_f32;
  cfg.dynamicSmemBytes = fused ? Plan::kAllocBytesEpi : Plan::kAllocBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e;
  if (b_layout == B200_B_KN) {
    e = fused ? cudaLaunchKernelEx(&cfg, b200::gemm_bf16_skinny_kernel<MPAD, stages, true, true>, tmB, tmA, tmC, p)
              : cudaLaunchKernelEx(&cfg, b200::gemm_bf16_skinny_kernel<MPAD, stages, true, false>, tmB, tmA, tmC, p);
  } else {
    e = fused ? cudaLaunchKernelEx(&cfg, b200::gemm_bf16_skinny_kernel<MPAD, stages, false, true>, tmB, tmA, tmC, p)
              : cudaLaunchKernelEx(&cfg, b200::gemm_bf16_skinny_kernel<MPAD, stages, false, false>, tmB, tmA, tmC, p);
  }
  return e == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

}  // namespace

namespace {

// The exchange's dependencies of one GEMM (b200_bcast_gemm): flags in this
// GPU's memory that must reach dep_value before B may be read, and flags in
// the writers' memory that get rel_value once B is no longer read.
struct PeerHooks {
  const uint32_t* dep[b200::kBcastMaxWorld];
  uint32_t* rel[b200::kBcastMaxWorld];
  uint32_t* counter;  // this GPU's count of CTA pairs done reading (pair kernel)
  int n_dep, n_rel;
  uint32_t dep_value, rel_value;
};

// Kernels without the in-kernel hooks take them as stream operations around
// the launch (the wait before, the release after).
int hooks_before(const PeerHooks* h, cudaStream_t stream) {
  for (int i = 0; h != nullptr && i < h->n_dep; ++i) {
    const int rc = b200_wait_u32(h->dep[i], h->dep_value, stream);
    if (rc != B200_OK) return rc;
  }
  return B200_OK;
}
int hooks_after(const PeerHooks* h, cudaStream_t stream) {
  for (int i = 0; h != nullptr && i < h->n_rel; ++i) {
    const int rc = b200_signal_u32(h->rel[i], h->rel_value, stream);
    if (rc != B200_OK) return rc;
  }
  return B200_OK;
}

// `epi` == nullptr: plain GEMM, C = bf16(A op(B)).  Otherwise a validated
// fused epilogue (see b200_gemm_bf16_ex); C is then D, of its element type.
// M > 128 problems so small that 256 x 256 CTA-pair tiles would occupy at
// most half of the SMs, while 128 x 64 single-CTA tiles fit in one wave:
// the small tiles spread the work over up to 4x more SMs (1024^3: 16 pairs
// = 32 SMs against 128 CTAs).
inline bool use_small_tiles(const DeviceState& st, int64_t M, int64_t N) {
  const int64_t pair_tiles = ((M + b200::kPairBM - 1) / b200::kPairBM) * ((N + kPairBN - 1) / kPairBN);
  const int64_t small_tiles = ((M + b200::kBM - 1) / b200::kBM) * ((N + kSmallBN - 1) / kSmallBN);
  return M > b200::kBM && 4 * pair_tiles <= st.sm_count && small_tiles <= st.sm_count;
}

// `outs` != nullptr: the gathering GEMM (b200_gemm_bf16_allgather): CTA-pair
// 256 x 256 tiles, every tile stored through each of outs->m[0 .. n_out).
// `hooks` != nullptr (M, N, K >= 1, no workspace): B is an exchange slot
// (b200_bcast_gemm); the pair kernel waits and releases inside, the others
// get stream operations around their launch.
int gemm_impl(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
              int64_t ldc, int b_layout, void* workspace, size_t workspace_bytes, void* stream_,
              const b200::EpilogueParams* epi_in = nullptr, const b200::OutMaps* outs = nullptr, int n_out = 1,
              const PeerHooks* hooks = nullptr) {
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARG;
  if (b_layout != B200_B_NK && b_layout != B200_B_KN) return B200_ERR_INVALID_ARG;
  const int64_t kLim = 0x7fffffffLL;
  if (M > kLim || N > kLim || K > kLim) return B200_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return B200_OK;
  if (C == nullptr) return B200_ERR_INVALID_ARG;
  if (ldc < N) return B200_ERR_INVALID_ARG;
  b200::EpilogueParams epi{};
  epi.alpha = 1.0f;
  if (epi_in != nullptr) epi = *epi_in;
  const bool f32 = epi.out_f32 != 0;
  if (!aligned16(C) || (ldc % (f32 ? 4 : 8)) != 0) return B200_ERR_ALIGNMENT;

  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);

  if (K == 0) {  // empty reduction: C = 0, in D's element type (bf16, or fp32 through the fused epilogue)
    if (epi.active) return B200_ERR_INVALID_ARG;  // bias / beta * C_in need K >= 1 (no kernel for K = 0)
    const size_t esize = f32 ? 4 : 2;
    return cudaMemset2DAsync(C, (size_t)ldc * esize, 0, (size_t)N * esize, (size_t)M, stream) == cudaSuccess
               ? B200_OK
               : B200_ERR_CUDA;
  }
  if (A == nullptr || B == nullptr) return B200_ERR_INVALID_ARG;
  if (lda < K) return B200_ERR_INVALID_ARG;
  if (ldb < (b_layout == B200_B_NK ? K : N)) return B200_ERR_INVALID_ARG;
  if (!aligned16(A) || !aligned16(B) || (lda % 8) != 0 || (ldb % 8) != 0) return B200_ERR_ALIGNMENT;

  // M <= 128: swap-AB split-K kernel (HBM-bound shapes).  Larger M: CTA pairs
  // on 256-row tiles, or single CTAs on 128 x 64 tiles for problems too
  // small to occupy the GPU with pairs (use_small_tiles).  (The single-CTA
  // 128 x 256 kernel remains for callers that force it with
  // b200_gemm_set_kernel.)
  const int force = outs != nullptr ? kForcePair : g_force_kernel.load(std::memory_order_relaxed);
  if (force == kForceSkinny && M > 128) return B200_ERR_INVALID_ARG;
  if (force == kForceSkinny || (force == kForceAuto && M <= 128)) {
    if ((rc = hooks_before(hooks, stream)) != B200_OK) return rc;
    if (M <= 16) rc = launch_skinny<16>(*st, A, B, C, M, N, K, lda, ldb, ldc, b_layout, epi, stream);
    else if (M <= 32) rc = launch_skinny<32>(*st, A, B, C, M, N, K, lda, ldb, ldc, b_layout, epi, stream);
    else if (M <= 64) rc = launch_skinny<64>(*st, A, B, C, M, N, K, lda, ldb, ldc, b_layout, epi, stream);
    else rc = launch_skinny<128>(*st, A, B, C, M, N, K, lda, ldb, ldc, b_layout, epi, stream);
    return rc == B200_OK ? hooks_after(hooks, stream) : rc;
  }
  const bool use_small = force == kForceAuto && use_small_tiles(*st, M, N);
  const bool use_pair = force == kForcePair || (force == kForceAuto && M > b200::kBM && !use_small);
  const int max_pairs = st->max_pairs;
  const int64_t m_blk_pair = (M + b200::kPairBM - 1) / b200::kPairBM;
  const int32_t k_blks = (int32_t)((K + b200::kBK - 1) / b200::kBK);
  // Split-K tail (only with a caller workspace) runs on 256 x 256 tiles.
  SplitPlan split{};
  bool use_split = false;
  if (use_pair && workspace != nullptr) {
    split = plan_split(m_blk_pair * ((N + kPairBN - 1) / kPairBN), k_blks, max_pairs, kPairBN);
    use_split = split.parts >= 2 && workspace_bytes >= split.bytes() &&
                (reinterpret_cast<uintptr_t>(workspace) % kWsAlign) == 0;
  }
  // Otherwise 256 x 512 tiles, unless they quantise worse onto the CTA pairs:
  // useful fraction of the launched waves, counting the unused columns of a
  // partial last tile.  The wide tile moves 25 % fewer operand bytes per FLOP,
  // so it may lose up to 3 % here (B200: 8192^3 +5 %, 16384^3 +11 %, but
  // 5000x4096x4096, 3 waves for 2.16 waves of work, -8 %).
  auto wave_eff = [&](int64_t bn_) {
    const int64_t n_blk = (N + bn_ - 1) / bn_;
    const int64_t t = m_blk_pair * n_blk;
    const int64_t rounds = (t + max_pairs - 1) / max_pairs;
    return ((double)t / (double)(rounds * max_pairs)) * ((double)N / (double)(n_blk * bn_));
  };
  // A fused epilogue does more work per tile (C_in loads, fp32 stores); the
  // wide tile's single TMEM accumulator would expose it, the 256-column
  // tiles' double-buffered accumulators hide it behind the next tile.
  const bool fused_epi = epi.active || epi.out_f32 || outs != nullptr;
  const bool use_wide = use_pair && !use_split && !fused_epi &&
                        m_blk_pair * ((N + kPairWideBN - 1) / kPairWideBN) >= max_pairs &&
                        wave_eff(kPairWideBN) >= 0.97 * wave_eff(kPairBN);
  const uint32_t bn = use_small   ? (uint32_t)kSmallBN
                      : !use_pair ? (uint32_t)kBN
                      : use_wide  ? (uint32_t)kPairWideBN
                                  : (uint32_t)kPairBN;
  // B rows (K-major) one TMA box covers: a pair CTA loads 128-column blocks.
  const uint32_t b_rows = use_pair ? 128u : bn;

  CUtensorMap tmA, tmB, tmC;
  if ((rc = encode_2d(&tmA, A, (uint64_t)K, (uint64_t)M, (uint64_t)lda, b200::kBK, b200::kBM, true)) != B200_OK)
    return rc;
  if (b_layout == B200_B_NK) {
    rc = encode_2d(&tmB, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, b200::kBK, b_rows, true);
  } else {
    rc = encode_2d(&tmB, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, 64, b200::kBK, true);
  }
  if (rc != B200_OK) return rc;
  // D store box: 32 rows of one warp x one 128-byte swizzle row (64 bf16 or
  // 32 fp32 columns).
  if ((rc = encode_2d(&tmC, C, (uint64_t)N, (uint64_t)M, (uint64_t)ldc, f32 ? 32u : (uint32_t)b200::kEpiCols,
                      b200::kEpiRowsPerWarp, false, true, f32)) != B200_OK)
    return rc;

  const int64_t bm = use_pair ? b200::kPairBM : b200::kBM;
  b200::GemmParams p{};
  p.M = (int32_t)M;
  p.N = (int32_t)N;
  p.K = (int32_t)K;
  p.num_m_blk = (int32_t)((M + bm - 1) / bm);
  p.num_n_blk = (int32_t)((N + bn - 1) / bn);
  p.num_k_blk = (int32_t)((K + b200::kBK - 1) / b200::kBK);
  const int64_t tiles = (int64_t)p.num_m_blk * p.num_n_blk;
  if (tiles > kLim) return B200_ERR_TOO_LARGE;
  p.num_tiles = (int32_t)tiles;
  p.group_m = kGroupM;
  p.b_mn_major = (b_layout == B200_B_KN) ? 1u : 0u;
  p.timeout_ns = st->timeout_ns;
  p.status = st->status_ptr;
  p.epi = epi;
  p.num_out = 1;

  if (!use_pair) {
    p.sk_first = p.num_work = p.num_tiles;
    p.sk_parts = 1;
    p.sk_kpp = p.num_k_blk;
    const int grid = (int)(tiles < st->sm_count ? tiles : st->sm_count);
    const bool fused = epi.active || epi.out_f32;
    using SingleKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const b200::GemmParams);
    static const SingleKernel kSingle[2][2][2] = {
        {{b200::gemm_bf16_tcgen05_kernel<kBN, kStages, false, false>,
          b200::gemm_bf16_tcgen05_kernel<kBN, kStages, false, true>},
         {b200::gemm_bf16_tcgen05_kernel<kBN, kStages, true, false>,
          b200::gemm_bf16_tcgen05_kernel<kBN, kStages, true, true>}},
        {{b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, false, false>,
          b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, false, true>},
         {b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, true, false>,
          b200::gemm_bf16_tcgen05_kernel<kSmallBN, kSmallStages, true, true>}}};
    const SingleKernel kern = kSingle[use_small ? 1 : 0][p.b_mn_major ? 1 : 0][fused ? 1 : 0];
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid, 1, 1);
    cfg.blockDim = dim3(b200::kNumThreads, 1, 1);
    cfg.dynamicSmemBytes = use_small ? b200::SmemPlan<kSmallBN, kSmallStages>::kAllocBytes
                                     : b200::SmemPlan<kBN, kStages>::kAllocBytes;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if ((rc = hooks_before(hooks, stream)) != B200_OK) return rc;
    if (cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmC, p) != cudaSuccess) return B200_ERR_CUDA;
    return hooks_after(hooks, stream);
  }
  p.sk_first = p.num_tiles;
  p.sk_parts = 1;
  p.sk_kpp = p.num_k_blk;
  p.num_work = p.num_tiles;
  if (use_split) {
    const SplitPlan& sp = split;
    {
      p.sk_first = sp.first;
      p.sk_parts = sp.parts;
      p.sk_kpp = sp.kpp;
      p.num_work = sp.work;
      p.workspace = static_cast<float*>(workspace);
      p.flags = reinterpret_cast<uint64_t*>(static_cast<char*>(workspace) + sp.partial_bytes);
      // The workspace is not initialised: a flag may hold anything.  A
      // 64-bit tag with a random per-process half makes an accidental match
      // with leftover memory contents practically impossible; the counter
      // half keeps consecutive launches apart.
      const uint32_t n = st->epoch.fetch_add(1, std::memory_order_relaxed) + 1;
      p.epoch = ((uint64_t)process_salt() << 32) | (uint64_t)n;
    }
  }
  if (hooks != nullptr) {
    // In the kernel: every producer waits for the dep flags before its first
    // load of B, and the last CTA pair to finish loading writes the releases.
    for (int i = 0; i < hooks->n_dep; ++i) p.dep_flags[i] = hooks->dep[i];
    for (int i = 0; i < hooks->n_rel; ++i) p.rel_flags[i] = hooks->rel[i];
    p.n_dep = hooks->n_dep;
    p.n_rel = hooks->n_rel;
    p.dep_value = hooks->dep_value;
    p.rel_value = hooks->rel_value;
    p.rel_counter = hooks->counter;
  }
  const int64_t work = p.num_work;
  const int pairs = (int)(work < max_pairs ? work : max_pairs);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(b200::kNumThreads, 1, 1);
  cfg.dynamicSmemBytes = use_wide ? b200::PairSmemPlan<kPairWideBN, kPairWideStages>::kAllocBytes
                                  : b200::PairSmemPlan<kPairBN, kPairStages>::kAllocBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // Pick the instantiation: tile width x B layout x (plain | fused epilogue).
  using PairKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const b200::GemmParams);
  static const PairKernel kPair[2][2][2] = {
      {{b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, false, false>,
        b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, false, true>},
       {b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, true, false>,
        b200::gemm_bf16_pair_kernel<kPairBN, kPairStages, true, true>}},
      {{b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, false, false>,
        b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, false, true>},
       {b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, true, false>,
        b200::gemm_bf16_pair_kernel<kPairWideBN, kPairWideStages, true, true>}}};
  const bool fused = epi.active || epi.out_f32;
  if (outs != nullptr) {
    p.num_out = n_out;
    const cudaError_t e =
        p.b_mn_major ? cudaLaunchKernelEx(&cfg, b200::gemm_bf16_pair_gather_kernel<true>, tmA, tmB, *outs, p)
                     : cudaLaunchKernelEx(&cfg, b200::gemm_bf16_pair_gather_kernel<false>, tmA, tmB, *outs, p);
    return e == cudaSuccess ? B200_OK : B200_ERR_CUDA;
  }
  PairKernel kern = kPair[use_wide ? 1 : 0][p.b_mn_major ? 1 : 0][fused ? 1 : 0];
  if (use_wide && !fused && st->wide8_regs_ok) {
    // Plain 256 x 512 tiles: eight epilogue warps free the accumulator from
    // registers (gemm_sm100_pair.cuh, kWide8Threads).
    kern = p.b_mn_major ? b200::gemm_bf16_pair_wide8_kernel<true> : b200::gemm_bf16_pair_wide8_kernel<false>;
    cfg.blockDim = dim3(b200::kWide8Threads, 1, 1);
  }
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmA, tmB, tmC, p);
  return e == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

}  // namespace

extern "C" B200_API int b200_gemm_bf16(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                       int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* stream) {
  return gemm_impl(A, B, C, M, N, K, lda, ldb, ldc, b_layout, nullptr, 0, stream);
}

extern "C" B200_API int b200_bcast_gemm(b200_bcast* b, int64_t step, size_t b_offset, const void* A, const void* B0,
                                        void* C, int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb,
                                        int64_t ldc, int b_layout, void* stream) {
  if (b == nullptr || step < 0) return B200_ERR_INVALID_ARG;
  if (b->world == 1 || b->rank == 0) return gemm_impl(A, B0, C, M, N, K, lda, ldb, ldc, b_layout, nullptr, 0, stream);
  if (M < 0 || N < 0 || K < 0 || b_layout < B200_B_NK || b_layout > B200_B_KN) return B200_ERR_INVALID_ARG;
  const int64_t b_rows = b_layout == B200_B_NK ? N : K;
  if (b_offset > b->nbytes ||
      (b_rows > 0 && ((uint64_t)(b_rows - 1) * (uint64_t)ldb + (uint64_t)(b_layout == B200_B_NK ? K : N)) * 2 >
                         (uint64_t)(b->nbytes - b_offset)))
    return B200_ERR_INVALID_ARG;  // B would run past this rank's slot
  const int slot = (int)(step % b200::kBcastSlots);
  PeerHooks h{};
  for (int r = 0; r < b->world; ++r) {
    if (r == b->rank) continue;
    h.dep[h.n_dep++] = b200::bcast_ready(b, b->rank, slot, r, b200::kBcastParts - 1);  // r's copies have landed
    h.rel[h.n_rel++] = b200::bcast_done(b, r, b->rank);        // each writer: this rank is done with the slot
  }
  h.counter = b200::bcast_counter(b);
  h.dep_value = h.rel_value = (uint32_t)(step + 1);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (M == 0 || N == 0 || K == 0) {  // nothing reads B: keep the protocol with stream operations
    int rc = hooks_before(&h, s);
    if (rc == B200_OK)
      rc = gemm_impl(A, b->slot[b->rank][slot] + b_offset, C, M, N, K, lda, ldb, ldc, b_layout, nullptr, 0, stream);
    return rc == B200_OK ? hooks_after(&h, s) : rc;
  }
  return gemm_impl(A, b->slot[b->rank][slot] + b_offset, C, M, N, K, lda, ldb, ldc, b_layout, nullptr, 0, stream,
                   nullptr, nullptr, 1, &h);
}

extern "C" B200_API int b200_gemm_bf16_ws(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                          int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  if (workspace == nullptr && workspace_bytes != 0) return B200_ERR_INVALID_ARG;
  if (workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) % kWsAlign) != 0) return B200_ERR_ALIGNMENT;
  return gemm_impl(A, B, C, M, N, K, lda, ldb, ldc, b_layout, workspace, workspace_bytes, stream);
}

extern "C" B200_API int b200_gemm_bf16_ex(const void* A, const void* B, void* D, int64_t M, int64_t N, int64_t K,
                                          int64_t lda, int64_t ldb, int64_t ldd, int b_layout, const b200_epilogue* epi,
                                          void* stream) {
  if (epi == nullptr) return gemm_impl(A, B, D, M, N, K, lda, ldb, ldd, b_layout, nullptr, 0, stream);
  if (epi->d_dtype != B200_DTYPE_BF16 && epi->d_dtype != B200_DTYPE_F32) return B200_ERR_INVALID_ARG;
  b200::EpilogueParams e{};
  e.alpha = epi->alpha;
  e.beta = epi->beta;
  e.out_f32 = epi->d_dtype == B200_DTYPE_F32 ? 1u : 0u;
  if (epi->bias != nullptr) {
    if (!aligned16(epi->bias)) return B200_ERR_ALIGNMENT;
    e.bias = static_cast<const __nv_bfloat16*>(epi->bias);
  }
  if (epi->beta != 0.0f) {
    if (epi->c_in == nullptr || epi->ldc_in < N) return B200_ERR_INVALID_ARG;
    if (!aligned16(epi->c_in) || (epi->ldc_in % 8) != 0) return B200_ERR_ALIGNMENT;
    // In place (C_in = D) only when D is bf16 with the same pitch: every
    // element is read before it is overwritten, by the thread that writes it.
    if (epi->c_in == D && (e.out_f32 || epi->ldc_in != ldd)) return B200_ERR_INVALID_ARG;
    e.c_in = static_cast<const __nv_bfloat16*>(epi->c_in);
    e.ldc_in = epi->ldc_in;
  }
  e.active = (e.alpha != 1.0f || e.beta != 0.0f || e.bias != nullptr) ? 1u : 0u;
  return gemm_impl(A, B, D, M, N, K, lda, ldb, ldd, b_layout, nullptr, 0, stream, &e);
}

extern "C" B200_API int b200_gemm_bf16_allgather(const void* A, const void* B, void* const* outputs,
                                                 int num_outputs, int64_t M_local, int64_t N, int64_t K, int64_t lda,
                                                 int64_t ldb, int64_t ldc, int64_t row0, int64_t M_total,
                                                 int b_layout, void* stream) {
  if (outputs == nullptr || num_outputs < 1 || num_outputs > b200::kMaxOutMaps) return B200_ERR_INVALID_ARG;
  if (M_local < 0 || N < 0 || K < 0 || row0 < 0 || M_total < 0 || row0 + M_local > M_total) {
    return B200_ERR_INVALID_ARG;
  }
  if (M_local == 0 || N == 0) return B200_OK;
  if (K == 0) return B200_ERR_INVALID_ARG;  // no kernel for an empty reduction here
  if (ldc < N) return B200_ERR_INVALID_ARG;
  if ((ldc % 8) != 0) return B200_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  b200::OutMaps outs{};
  for (int i = 0; i < num_outputs; ++i) {
    if (outputs[i] == nullptr || !aligned16(outputs[i])) return B200_ERR_ALIGNMENT;
    // Every output must be device memory this process can address (a local
    // buffer or a peer's buffer opened with b200_ipc_open).
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, outputs[i]) != cudaSuccess || at.type != cudaMemoryTypeDevice) {
      cudaGetLastError();
      return B200_ERR_INVALID_ARG;
    }
    // This rank's rows of rank i's gathered C: a [M_local, N] view starting
    // at row row0, so that TMA clips the last tile at M_local.
    const char* base = static_cast<const char*>(outputs[i]) + (size_t)row0 * (size_t)ldc * 2;
    if ((rc = encode_2d(&outs.m[i], base, (uint64_t)N, (uint64_t)M_local, (uint64_t)ldc, b200::kEpiCols,
                        b200::kEpiRowsPerWarp, false)) != B200_OK)
      return rc;
  }
  void* C0 = static_cast<char*>(outputs[0]) + (size_t)row0 * (size_t)ldc * 2;
  return gemm_impl(A, B, C0, M_local, N, K, lda, ldb, ldc, b_layout, nullptr, 0, stream, nullptr, &outs,
                   num_outputs);
}

extern "C" B200_API int b200_ipc_alloc(size_t bytes, void** dev_ptr, void* handle) {
  if (dev_ptr == nullptr || handle == nullptr || bytes == 0) return B200_ERR_INVALID_ARG;
  *dev_ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_CUDA;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return B200_ERR_CUDA;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == B200_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return B200_OK;
}

extern "C" B200_API int b200_ipc_free(void* dev_ptr) {
  return cudaFree(dev_ptr) == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" B200_API int b200_ipc_open(const void* handle, void** dev_ptr) {
  if (dev_ptr == nullptr || handle == nullptr) return B200_ERR_INVALID_ARG;
  *dev_ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_CUDA;
  }
  *dev_ptr = p;
  return B200_OK;
}

extern "C" B200_API int b200_ipc_close(void* dev_ptr) {
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

namespace {

// Workspace layout of b200_gemm_f32: A' [M, ldk6] then B' ([N, ldk6] or
// [6K, ldn]), bf16, each 256-byte aligned; ldk6 = 6K rounded up to 8.
struct F32Plan {
  int64_t ldk6, ld_b;
  size_t a_bytes, b_bytes;
  size_t total() const { return a_bytes + b_bytes; }
};

inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

F32Plan plan_f32(int64_t M, int64_t N, int64_t K, int b_layout) {
  F32Plan f{};
  f.ldk6 = (6 * K + 7) / 8 * 8;
  f.a_bytes = round_up((size_t)M * (size_t)f.ldk6 * 2, 256);
  if (b_layout == B200_B_NK) {
    f.ld_b = f.ldk6;
    f.b_bytes = round_up((size_t)N * (size_t)f.ldk6 * 2, 256);
  } else {
    f.ld_b = (N + 7) / 8 * 8;
    f.b_bytes = round_up((size_t)6 * (size_t)K * (size_t)f.ld_b * 2, 256);
  }
  return f;
}

int launch_split(const float* src, int64_t rows, int64_t cols, int64_t ld_src, uint16_t* dst, int64_t ld_dst,
                 int64_t seg_off, uint32_t order, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return B200_OK;
  const unsigned gx = (unsigned)std::min<int64_t>((cols + 255) / 256, 64);
  const unsigned gy = (unsigned)std::min<int64_t>(rows, 8192);
  b200::split_f32_bf16x3_kernel<<<dim3(gx, gy), 256, 0, stream>>>(src, rows, cols, ld_src, dst, ld_dst, seg_off,
                                                                    order);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

}  // namespace

extern "C" B200_API int b200_gemm_f32_workspace_bytes(int64_t M, int64_t N, int64_t K, int b_layout, size_t* bytes) {
  if (bytes == nullptr || M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARG;
  if (b_layout != B200_B_NK && b_layout != B200_B_KN) return B200_ERR_INVALID_ARG;
  *bytes = (M == 0 || N == 0 || K == 0) ? 0 : plan_f32(M, N, K, b_layout).total();
  return B200_OK;
}

extern "C" B200_API int b200_gemm_f32(const float* A, const float* B, float* C, int64_t M, int64_t N, int64_t K,
                                      int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* workspace,
                                      size_t workspace_bytes, void* stream_) {
  if (M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARG;
  if (b_layout != B200_B_NK && b_layout != B200_B_KN) return B200_ERR_INVALID_ARG;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || 6 * K > 0x7fffffffLL) return B200_ERR_TOO_LARGE;
  if (M == 0 || N == 0) return B200_OK;
  if (C == nullptr || ldc < N) return B200_ERR_INVALID_ARG;
  if (!aligned16(C) || (ldc % 4) != 0) return B200_ERR_ALIGNMENT;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  if (K == 0) {  // empty reduction: C = 0
    DeviceState* st = nullptr;
    const int rc = current_device_state(&st);
    if (rc != B200_OK) return rc;
    return cudaMemset2DAsync(C, (size_t)ldc * 4, 0, (size_t)N * 4, (size_t)M, stream) == cudaSuccess
               ? B200_OK
               : B200_ERR_CUDA;
  }
  if (A == nullptr || B == nullptr || lda < K || ldb < (b_layout == B200_B_NK ? K : N)) return B200_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(A) & 3u) || (reinterpret_cast<uintptr_t>(B) & 3u)) return B200_ERR_ALIGNMENT;
  const F32Plan f = plan_f32(M, N, K, b_layout);
  if (workspace == nullptr || workspace_bytes < f.total()) return B200_ERR_INVALID_ARG;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return B200_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  uint16_t* Ap = static_cast<uint16_t*>(workspace);
  uint16_t* Bp = reinterpret_cast<uint16_t*>(static_cast<char*>(workspace) + f.a_bytes);
  if ((rc = launch_split(A, M, K, lda, Ap, f.ldk6, K, b200::kSplitOrderA, stream)) != B200_OK) return rc;
  if (b_layout == B200_B_NK) {
    rc = launch_split(B, N, K, ldb, Bp, f.ld_b, K, b200::kSplitOrderB, stream);
  } else {
    rc = launch_split(B, K, N, ldb, Bp, f.ld_b, K * f.ld_b, b200::kSplitOrderB, stream);
  }
  if (rc != B200_OK) return rc;
  b200::EpilogueParams e{};
  e.alpha = 1.0f;
  e.out_f32 = 1u;
  return gemm_impl(Ap, Bp, C, M, N, 6 * K, f.ldk6, f.ld_b, ldc, b_layout, nullptr, 0, stream, &e);
}

namespace {

// 3-D bf16 tensor map {cols, rows, batch} over a [batch, rows, ld] array,
// 128B swizzle; rows clip per batch.
int encode_3d(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows, uint64_t batch, uint64_t ld_elems,
              uint32_t box_cols, uint32_t box_rows, bool is_load) {
  cuuint64_t dims[3] = {cols, rows, batch};
  cuuint64_t strides[2] = {ld_elems * 2, ld_elems * 2 * rows};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(ptr), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              is_load ? CU_TENSOR_MAP_L2_PROMOTION_L2_256B : CU_TENSOR_MAP_L2_PROMOTION_NONE,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_TENSOR_MAP;
}

}  // namespace

extern "C" B200_API int b200_flash_attn_bf16(const void* Q, const void* K, const void* V, void* O, int64_t batch,
                                             int64_t seq_len, int64_t heads, int64_t kv_heads,
                                             int64_t head_dim, int causal, void* stream_) {
  if (batch < 0 || seq_len < 0 || heads < 0 || kv_heads < 0) return B200_ERR_INVALID_ARG;
  if (head_dim != b200::kAttnD) return B200_ERR_INVALID_ARG;
  if ((heads > 0 && kv_heads == 0) || (kv_heads > 0 && heads % kv_heads != 0)) return B200_ERR_INVALID_ARG;
  if (batch == 0 || seq_len == 0 || heads == 0) return B200_OK;
  if (batch > 65535 || heads > 65535 || heads * batch > 0x7fffffffLL || seq_len > 65535LL * 2 * b200::kAttnBQ ||
      heads * head_dim > 0x7fffffffLL)
    return B200_ERR_TOO_LARGE;
  if (Q == nullptr || K == nullptr || V == nullptr || O == nullptr) return B200_ERR_INVALID_ARG;
  if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O)) return B200_ERR_ALIGNMENT;
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  if (!st->attn_regs_ok) return B200_ERR_CUDA;  // built with another register count: never launch it
  const uint64_t cols = (uint64_t)(heads * head_dim);
  const uint64_t kv_cols = (uint64_t)(kv_heads * head_dim);
  // The CTA-pair kernel (each SM reading half of every K and V tile) only
  // when asked for: on B200 it measured slower than the one-CTA kernel at
  // every size (attn_sm100_pair.cuh).
  const bool pair = g_attn_kernel.load(std::memory_order_relaxed) == B200_ATTN_KERNEL_PAIR;
  if (pair && !st->attn_pair_regs_ok) return B200_ERR_CUDA;  // built with another register count
  if (pair && 2 * heads * batch > 0x7fffffffLL) return B200_ERR_TOO_LARGE;
  CUtensorMap tmQ, tmK, tmV, tmO;
  if ((rc = encode_3d(&tmQ, Q, cols, (uint64_t)seq_len, (uint64_t)batch, cols, 64, 128, true)) != B200_OK ||
      (rc = encode_3d(&tmK, K, kv_cols, (uint64_t)seq_len, (uint64_t)batch, kv_cols, 64, pair ? 64 : 128, true)) !=
          B200_OK ||
      (rc = encode_3d(&tmV, V, kv_cols, (uint64_t)seq_len, (uint64_t)batch, kv_cols, 64, 64, true)) != B200_OK ||
      (rc = encode_3d(&tmO, O, cols, (uint64_t)seq_len, (uint64_t)batch, cols, 64, 32, false)) != B200_OK)
    return rc;
  b200::AttnParams p{};
  p.seq_len = (int32_t)seq_len;
  p.heads = (int32_t)heads;
  p.batch = (int32_t)batch;
  p.group = (int32_t)(heads / kv_heads);
  p.num_q_tiles = (int32_t)((seq_len + b200::kAttnBQ - 1) / b200::kAttnBQ);
  p.causal = causal ? 1u : 0u;
  {
    // With a causal mask, pairing a short row with a long one evens out the
    // CTAs' work; that only pays while the whole grid runs in one wave (with
    // more waves, longest-first order balances the SMs better).
    const int64_t pairs = (p.num_q_tiles + b200::kAttnQTiles - 1) / b200::kAttnQTiles;
    p.balanced = (causal && p.num_q_tiles > 2 && pairs * heads * batch <= st->sm_count) ? 1u : 0u;
  }
  p.scale_log2 = 1.4426950408889634f / sqrtf((float)head_dim);
  p.timeout_ns = st->timeout_ns;
  p.status = st->status_ptr;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  if (pair) {
    p.balanced = 0u;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 2;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.gridDim = dim3((unsigned)(2 * heads * batch), (unsigned)((p.num_q_tiles + 3) / 4), 1);
    cfg.blockDim = dim3(b200::kAttnThreads, 1, 1);
    cfg.dynamicSmemBytes = b200::AttnPairSmemPlan::kAllocBytes;
    cfg.stream = reinterpret_cast<cudaStream_t>(stream_);
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, b200::flash_attn_fwd_pair_kernel, tmQ, tmK, tmV, tmO, p) == cudaSuccess
               ? B200_OK
               : B200_ERR_CUDA;
  }
  cfg.gridDim = dim3((unsigned)(heads * batch), (unsigned)((p.num_q_tiles + b200::kAttnQTiles - 1) / b200::kAttnQTiles),
                     1);
  cfg.blockDim = dim3(b200::kAttnThreads, 1, 1);
  cfg.dynamicSmemBytes = b200::AttnSmemPlan::kAllocBytes;
  cfg.stream = reinterpret_cast<cudaStream_t>(stream_);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, b200::flash_attn_fwd_kernel, tmQ, tmK, tmV, tmO, p) == cudaSuccess ? B200_OK
                                                                                                      : B200_ERR_CUDA;
}

namespace {
// The split-K plan gemm_impl would use for this shape when given a large
// enough workspace: the same kernel choice (forced kernel, small-tile path,
// M <= 128) and the same plan.  parts < 2: no split, no scratch.
SplitPlan planned_split(const DeviceState& st, int64_t M, int64_t N, int64_t K) {
  SplitPlan none{};
  none.parts = 1;
  if (M <= 0 || N <= 0 || K <= 0) return none;
  const int force = g_force_kernel.load(std::memory_order_relaxed);
  const bool pair = force == kForcePair || (force == kForceAuto && M > b200::kBM && !use_small_tiles(st, M, N));
  if (!pair) return none;
  const int64_t tiles = ((M + b200::kPairBM - 1) / b200::kPairBM) * ((N + kPairBN - 1) / kPairBN);
  return plan_split(tiles, (int32_t)((K + b200::kBK - 1) / b200::kBK), st.max_pairs, kPairBN);
}
}  // namespace

extern "C" B200_API int b200_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K, int b_layout, size_t* bytes) {
  if (bytes == nullptr || M < 0 || N < 0 || K < 0) return B200_ERR_INVALID_ARG;
  if (b_layout != B200_B_NK && b_layout != B200_B_KN) return B200_ERR_INVALID_ARG;
  *bytes = 0;
  DeviceState* st = nullptr;
  const int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  const SplitPlan sp = planned_split(*st, M, N, K);
  if (sp.parts >= 2) *bytes = sp.bytes();
  return B200_OK;
}

extern "C" B200_API int b200_gemm_status(void* stream_, uint32_t* device_bits) {
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  uint32_t bits = 0;
  const uint32_t zero = 0;
  if (cudaMemcpyAsync(&bits, st->status_ptr, sizeof(bits), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
    return B200_ERR_CUDA;
  if (cudaMemcpyAsync(st->status_ptr, &zero, sizeof(zero), cudaMemcpyHostToDevice, stream) != cudaSuccess)
    return B200_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return B200_ERR_CUDA;
  if (device_bits != nullptr) *device_bits = bits;
  return bits == 0 ? B200_OK : B200_ERR_DEVICE_TIMEOUT;
}

extern "C" B200_API int b200_gemm_set_timeout_ns(uint64_t timeout_ns) {
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  st->timeout_ns = timeout_ns == 0 ? kDefaultTimeoutNs : timeout_ns;
  return B200_OK;
}

namespace {
// One CTA waits, with the library's bounded wait, on an mbarrier that nothing
// ever arrives at.  The wait must give up after `timeout_ns` and report it in
// the status word — the same path a GEMM kernel takes when a role stalls.
__global__ void selftest_wait_timeout_kernel(uint64_t timeout_ns, uint32_t* status) {
#if B200_NO_SM100A_FEATURES
  if (threadIdx.x == 0 && status != nullptr) atomicOr(status, (uint32_t)b200::kDevWrongArch);
#else
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t abort_flag;
  if (threadIdx.x == 0) {
    b200::mbar_init(b200::smem_u32(&bar), 1);
    abort_flag = 0u;
    b200::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (!b200::mbar_wait(b200::smem_u32(&bar), 0u, timeout_ns, &abort_flag)) {
      atomicOr(status, (uint32_t)b200::kDevTimeoutMma);
    }
  }
#endif
}
}  // namespace

extern "C" B200_API int b200_gemm_selftest_wait_timeout(uint64_t timeout_ns, void* stream_) {
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) return B200_ERR_INVALID_ARG;
  selftest_wait_timeout_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream_)>>>(timeout_ns, st->status_ptr);
  return cudaGetLastError() == cudaSuccess ? B200_OK : B200_ERR_CUDA;
}

extern "C" B200_API int b200_flash_attn_set_kernel(int which) {
  if (which < B200_ATTN_KERNEL_AUTO || which > B200_ATTN_KERNEL_PAIR) return B200_ERR_INVALID_ARG;
  g_attn_kernel.store(which, std::memory_order_relaxed);
  return B200_OK;
}

extern "C" B200_API int b200_gemm_set_kernel(int which) {
  if (which < kForceAuto || which > kForceSkinny) return B200_ERR_INVALID_ARG;
  g_force_kernel.store(which, std::memory_order_relaxed);
  return B200_OK;
}

extern "C" B200_API const char* b200_gemm_strerror(int code) {
  switch (code) {
    case B200_OK: return "ok";
    case B200_ERR_INVALID_ARG: return "invalid argument";
    case B200_ERR_ALIGNMENT: return "pointer or row pitch not 16-byte aligned";
    case B200_ERR_UNSUPPORTED_DEVICE: return "current device is not sm_100 (B200)";
    case B200_ERR_CUDA: return "CUDA runtime call failed";
    case B200_ERR_TENSOR_MAP: return "tensor map encode failed";
    case B200_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case B200_ERR_TOO_LARGE: return "dimension too large";
    case B200_ERR_SCRATCH_LIMIT: return "split-K scratch needed exceeds the 16 MiB static buffer of b200_gemm_bf16_noalloc";
    default: return "unknown error";
  }
}

extern "C" B200_API const char* b200_gemm_version(void) { return "b200_gemm 0.1.0 sm_100a"; }

// ---------------------------------------------------------------------------
// Allocation-free variant of the split-K GEMM.
//
// Some callers cannot allocate device memory at the point where they multiply:
// a serving engine that reserves every byte of HBM at start-up and must not
// call cudaMalloc on its request path (cudaMalloc can synchronise the device
// and stall every stream), or a plugin whose host framework hands it raw
// buffers but no allocator.  For them the split-K scratch lives in a static
// device array inside this library instead of a caller workspace.
// ---------------------------------------------------------------------------
namespace {

// Static split-K scratch: 16 MiB, enough for any shape on a 148-SM B200.
// There a launch holds at most 74 CTA pairs; a split plan over `rem` leftover
// tiles in `parts` parts keeps rem x (parts - 1) x 2 partial tiles of
// 128 x 256 fp32 (128 KiB each) plus one 8-byte flag per partial, and the
// largest case, rem = 9 tiles in 8 parts, needs 126 partials = 15.75 MiB
// plus 1 KiB of flags (the compile-time check below recomputes it).
// Every GPU that loads this library holds it until the process exits.
constexpr size_t kNoAllocScratchBytes = 16u << 20;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Largest SplitPlan::bytes() plan_split can return for `pairs` CTA pairs and
// 256-column tiles (every rem in [1, pairs), parts = min(pairs / rem, 8)).
constexpr size_t max_split_bytes(int pairs) {
  size_t best = 0;
  for (int rem = 1; rem < pairs; ++rem) {
    const int parts = pairs / rem < 8 ? pairs / rem : 8;
    if (parts < 2) continue;
    const size_t slots = (size_t)rem * (size_t)(parts - 1) * 2;
    const size_t partial = (slots * (size_t)b200::kBM * (size_t)kPairBN * 4 + kWsAlign - 1) / kWsAlign * kWsAlign;
    const size_t flags = (slots * 8 + kWsAlign - 1) / kWsAlign * kWsAlign;
    if (partial + flags > best) best = partial + flags;
  }
  return best;
}
static_assert(max_split_bytes(74) <= kNoAllocScratchBytes,
              "the static scratch must hold every split plan of a 148-SM B200 (74 CTA pairs)");

// Scratch bytes the split plan of this shape needs (0 when it does not split).
size_t sp_needs(const DeviceState& st, int64_t M, int64_t N, int64_t K) {
  const SplitPlan sp = planned_split(st, M, N, K);
  return sp.parts >= 2 ? sp.bytes() : 0;
}

struct NoAllocState {
  std::once_flag once;
  int rc = B200_OK;
  void* scratch = nullptr;  // device address of g_noalloc_scratch on this device
};
NoAllocState g_noalloc[kMaxDevices];

}  // namespace

extern "C" B200_API int b200_gemm_bf16_noalloc(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                                               int64_t lda, int64_t ldb, int64_t ldc, int b_layout, void* stream) {
  DeviceState* st = nullptr;
  int rc = current_device_state(&st);
  if (rc != B200_OK) return rc;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
  // One-time set-up per device (runs inside the first call on that device,
  // with that device current): the host-side name g_noalloc_scratch is not a
  // device address, so look the address up and keep it.
  NoAllocState& na = g_noalloc[dev];
  std::call_once(na.once, [&] {
    na.rc = cudaGetSymbolAddress(&na.scratch, g_noalloc_scratch) == cudaSuccess ? B200_OK : B200_ERR_CUDA;
  });
  if (na.rc != B200_OK) return na.rc;
  // Reject shapes whose split-K scratch would not fit the static buffer
  // (none on a 148-SM B200; a device with more co-resident CTA pairs could
  // ask for more).  The plan is the one gemm_impl itself will choose, so the
  // check follows the same kernel selection; an error is returned rather
  // than a silent unsplit run, so a caller never gets a different summation
  // order than b200_gemm_bf16_ws would give for the same shape.
  if (sp_needs(*st, M, N, K) > kNoAllocScratchBytes) return B200_ERR_SCRATCH_LIMIT;
  // Nothing in the scratch needs clearing between calls: every partial tile is
  // written in full before it is read, and the hand-off flags are matched
  // against a tag that is new for every launch.
  return gemm_impl(A, B, C, M, N, K, lda, ldb, ldc, b_layout, na.scratch, kNoAllocScratchBytes, stream);
}
