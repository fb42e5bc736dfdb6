// Copy engines and stream-ordered flags between GPUs (C ABI in
// include/b200_gemm.h): the primitives the multi-GPU driver uses to move B
// from rank to rank over NVLink while the GEMM of the previous step holds
// every SM.
//
// A collective kernel (NCCL) needs SMs, and a persistent GEMM occupies all of
// them, so a broadcast queued beside the GEMM only runs between GEMMs.  Here
// the data moves with cudaMemcpyAsync between this GPU's memory and a peer's
// buffer mapped through CUDA IPC (the copy engines, no SMs), and readiness is
// signalled with stream memory operations: a 32-bit flag written into the
// reader's memory after the copy in the writer's stream, and a stream that
// waits for the flag before the kernel that reads the data.  Neither runs on
// an SM.  The driver entry points are fetched through the runtime, so
// nothing links against libcuda.
//
// The reference has no multi-GPU code; these have no counterpart there.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <mutex>
#include <new>

#include "b200_gemm.h"
#include "peer_bcast.h"

namespace {

std::once_flag g_memop_once;
PFN_cuStreamWriteValue32_v11070 g_write32 = nullptr;
PFN_cuStreamWaitValue32_v11070 g_wait32 = nullptr;

void load_memops() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPointByVersion("cuStreamWriteValue32", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_write32 = reinterpret_cast<PFN_cuStreamWriteValue32_v11070>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPointByVersion("cuStreamWaitValue32", &fn, 12000, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_wait32 = reinterpret_cast<PFN_cuStreamWaitValue32_v11070>(fn);
}

bool memops_ready() {
  std::call_once(g_memop_once, load_memops);
  return g_write32 != nullptr && g_wait32 != nullptr;
}

inline bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace

extern "C" B200_API int b200_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return B200_OK;
  if (dst == nullptr || src == nullptr) return B200_ERR_INVALID_ARG;
  if (cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)) !=
      cudaSuccess) {
    cudaGetLastError();
    return B200_ERR_CUDA;
  }
  return B200_OK;
}

extern "C" B200_API int b200_signal_u32(void* flag, uint32_t value, void* stream) {
  if (flag == nullptr || !aligned4(flag)) return B200_ERR_INVALID_ARG;
  if (!memops_ready()) return B200_ERR_CUDA;
  // Default flags: the write is ordered after (and made visible after) all
  // earlier work in the stream, including copies into the flag owner's memory.
  const CUresult r = g_write32(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag), value,
                               CU_STREAM_WRITE_VALUE_DEFAULT);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_CUDA;
}

extern "C" B200_API int b200_wait_u32(const void* flag, uint32_t value, void* stream) {
  if (flag == nullptr || !aligned4(flag)) return B200_ERR_INVALID_ARG;
  if (!memops_ready()) return B200_ERR_CUDA;
  // Later work in the stream starts once (int32_t)(*flag - value) >= 0.
  const CUresult r = g_wait32(reinterpret_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(const_cast<void*>(flag)),
                              value, CU_STREAM_WAIT_VALUE_GEQ);
  return r == CUDA_SUCCESS ? B200_OK : B200_ERR_CUDA;
}

// ---------------------------------------------------------------------------
// Per-step broadcast from rank 0 over the copy engines (b200_bcast_*): the
// protocol the multi-GPU driver runs every step, in native code so that a
// step costs three calls however many ranks there are.
//
// Every rank owns kSlots receive slots of `nbytes` (step s uses slot
// s % kSlots) and a flag array, all mapped by every peer (CUDA IPC).  Flags
// (uint32): ready[slot][sender][part] — that part of the sender's piece of
// that slot has landed (value step + 1); done[rank] — that rank has finished
// reading its slot of a step (value step + 1).  Pieces: the buffer is cut
// into world - 1 pieces (b200_bcast_piece), each moved in kBcastParts parts;
// rank 0 sends piece q-1 to rank q, and rank q forwards each part to every
// other receiving rank as soon as it has landed, so every byte leaves rank 0
// once and forwarding overlaps sending.  Copies to different peers go on
// different streams (different copy engines), so they run at the same time.  Before writing into a peer's slot for step s, a writer waits
// until that peer is done with step s - kSlots, which used the same slot.
// ---------------------------------------------------------------------------
namespace {
using b200::kBcastMaxWorld;
using b200::kBcastParts;
using b200::kBcastSlots;
inline uint32_t* ready_flag(const b200_bcast* b, int owner, int slot, int sender, int part) {
  return b200::bcast_ready(b, owner, slot, sender, part);
}
inline uint32_t* done_flag(const b200_bcast* b, int owner, int r) { return b200::bcast_done(b, owner, r); }
// Part k of a piece [off, off + len): 256-byte aligned starts.
inline void piece_part(size_t off, size_t len, int k, size_t* poff, size_t* plen) {
  auto bound = [&](int i) -> size_t {
    if (i >= kBcastParts) return off + len;
    size_t x = off + (len * (size_t)i / kBcastParts + 255) / 256 * 256;
    return x < off + len ? x : off + len;
  };
  *poff = bound(k);
  *plen = bound(k + 1) - *poff;
}
}  // namespace

extern "C" B200_API int b200_bcast_piece(int world, size_t nbytes, int index, size_t* offset, size_t* length) {
  if (offset == nullptr || length == nullptr || world < 2 || index < 0 || index >= world - 1)
    return B200_ERR_INVALID_ARG;
  const size_t parts = (size_t)(world - 1);
  auto bound = [&](size_t i) -> size_t {
    if (i >= parts) return nbytes;
    size_t b = (nbytes * i / parts + 255) / 256 * 256;
    return b < nbytes ? b : nbytes;
  };
  *offset = bound((size_t)index);
  *length = bound((size_t)index + 1) - *offset;
  return B200_OK;
}

extern "C" B200_API size_t b200_bcast_flag_bytes(int world) { return b200::bcast_flag_words(world) * sizeof(uint32_t); }

extern "C" B200_API int b200_bcast_create(int rank, int world, size_t nbytes, void* const* slots, void* const* flags,
                                          b200_bcast** out) {
  if (out == nullptr || slots == nullptr || flags == nullptr) return B200_ERR_INVALID_ARG;
  *out = nullptr;
  if (world < 1 || world > kBcastMaxWorld || rank < 0 || rank >= world) return B200_ERR_INVALID_ARG;
  b200_bcast* b = new (std::nothrow) b200_bcast{};
  if (b == nullptr) return B200_ERR_CUDA;
  b->rank = rank;
  b->world = world;
  b->nbytes = nbytes;
  for (int r = 0; r < world; ++r) {
    for (int k = 0; k < kBcastSlots; ++k) b->slot[r][k] = static_cast<char*>(slots[r * kBcastSlots + k]);
    b->flags[r] = static_cast<char*>(flags[r]);
    if (b->flags[r] == nullptr || !aligned4(b->flags[r])) {
      delete b;
      return B200_ERR_INVALID_ARG;
    }
  }
  bool ok = cudaEventCreateWithFlags(&b->start_ev, cudaEventDisableTiming) == cudaSuccess;
  for (int r = 0; ok && r < world; ++r) {
    ok = cudaStreamCreateWithFlags(&b->peer_stream[r], cudaStreamNonBlocking) == cudaSuccess &&
         cudaEventCreateWithFlags(&b->done_ev[r], cudaEventDisableTiming) == cudaSuccess;
  }
  if (!ok) {
    cudaGetLastError();
    b200_bcast_destroy(b);
    return B200_ERR_CUDA;
  }
  *out = b;
  return B200_OK;
}

extern "C" B200_API void b200_bcast_destroy(b200_bcast* b) {
  if (b == nullptr) return;
  for (int r = 0; r < b->world; ++r) {
    if (b->peer_stream[r] != nullptr) cudaStreamDestroy(b->peer_stream[r]);
    if (b->done_ev[r] != nullptr) cudaEventDestroy(b->done_ev[r]);
  }
  if (b->start_ev != nullptr) cudaEventDestroy(b->start_ev);
  delete b;
}

extern "C" B200_API int b200_bcast_issue(b200_bcast* b, int64_t step, const void* src, void* stream) {
  if (b == nullptr) return B200_ERR_INVALID_ARG;
  return b200_bcast_issue_range(b, step, src, 0, b->nbytes, stream);
}

extern "C" B200_API int b200_bcast_issue_range(b200_bcast* b, int64_t step, const void* src, size_t offset,
                                               size_t length, void* stream) {
  if (b == nullptr || step < 0) return B200_ERR_INVALID_ARG;
  if (offset > b->nbytes || length > b->nbytes - offset || (offset & 255u) != 0) return B200_ERR_INVALID_ARG;
  if (b->world == 1) return B200_OK;
  const int slot = (int)(step % kBcastSlots);
  const uint32_t v = (uint32_t)(step + 1);
  const bool reuse = step >= kBcastSlots;  // the slot held step - kSlots: wait until its reader is done
  const uint32_t v_prev = (uint32_t)(step - kBcastSlots + 1);
  int rc;
  // Every destination gets its own copy stream, started after the work
  // already on `stream` (rank 0's source is ready) and joined back into it.
  if (cudaEventRecord(b->start_ev, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return B200_ERR_CUDA;
  auto fork = [&](int dst) -> void* {
    return cudaStreamWaitEvent(b->peer_stream[dst], b->start_ev, 0) == cudaSuccess ? (void*)b->peer_stream[dst]
                                                                                    : nullptr;
  };
  auto join = [&](int dst) -> int {
    if (cudaEventRecord(b->done_ev[dst], b->peer_stream[dst]) != cudaSuccess ||
        cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), b->done_ev[dst], 0) != cudaSuccess)
      return B200_ERR_CUDA;
    return B200_OK;
  };
  if (b->rank == 0) {
    if (src == nullptr) return B200_ERR_INVALID_ARG;
    for (int q = 1; q < b->world; ++q) {
      void* ps = fork(q);
      if (ps == nullptr) return B200_ERR_CUDA;
      size_t off, len;
      if ((rc = b200_bcast_piece(b->world, length, q - 1, &off, &len)) != B200_OK) return rc;
      if (reuse && (rc = b200_wait_u32(done_flag(b, 0, q), v_prev, ps)) != B200_OK) return rc;
      for (int k = 0; k < kBcastParts; ++k) {
        size_t poff, plen;
        piece_part(offset + off, len, k, &poff, &plen);
        if ((rc = b200_copy_async(b->slot[q][slot] + poff, static_cast<const char*>(src) + poff, plen, ps)) != B200_OK)
          return rc;
        if ((rc = b200_signal_u32(ready_flag(b, q, slot, 0, k), v, ps)) != B200_OK) return rc;
      }
      if ((rc = join(q)) != B200_OK) return rc;
    }
    return B200_OK;
  }
  size_t off, len;
  if ((rc = b200_bcast_piece(b->world, length, b->rank - 1, &off, &len)) != B200_OK) return rc;
  for (int r = 1; r < b->world; ++r) {
    if (r == b->rank) continue;
    void* ps = fork(r);
    if (ps == nullptr) return B200_ERR_CUDA;
    if (reuse && (rc = b200_wait_u32(done_flag(b, b->rank, r), v_prev, ps)) != B200_OK) return rc;
    for (int k = 0; k < kBcastParts; ++k) {
      size_t poff, plen;
      piece_part(offset + off, len, k, &poff, &plen);
      // part k of my piece has landed: pass it on
      if ((rc = b200_wait_u32(ready_flag(b, b->rank, slot, 0, k), v, ps)) != B200_OK) return rc;
      if ((rc = b200_copy_async(b->slot[r][slot] + poff, b->slot[b->rank][slot] + poff, plen, ps)) != B200_OK)
        return rc;
      if ((rc = b200_signal_u32(ready_flag(b, r, slot, b->rank, k), v, ps)) != B200_OK) return rc;
    }
    if ((rc = join(r)) != B200_OK) return rc;
  }
  return B200_OK;
}

extern "C" B200_API int b200_bcast_wait(b200_bcast* b, int64_t step, void* stream) {
  if (b == nullptr || step < 0) return B200_ERR_INVALID_ARG;
  if (b->world == 1 || b->rank == 0) return B200_OK;
  const int slot = (int)(step % kBcastSlots);
  for (int r = 0; r < b->world; ++r) {
    if (r == b->rank) continue;
    const int rc = b200_wait_u32(ready_flag(b, b->rank, slot, r, kBcastParts - 1), (uint32_t)(step + 1), stream);
    if (rc != B200_OK) return rc;
  }
  return B200_OK;
}

extern "C" B200_API int b200_bcast_release(b200_bcast* b, int64_t step, void* stream) {
  if (b == nullptr || step < 0) return B200_ERR_INVALID_ARG;
  if (b->world == 1 || b->rank == 0) return B200_OK;
  for (int r = 0; r < b->world; ++r) {
    if (r == b->rank) continue;
    const int rc = b200_signal_u32(done_flag(b, r, b->rank), (uint32_t)(step + 1), stream);
    if (rc != B200_OK) return rc;
  }
  return B200_OK;
}
