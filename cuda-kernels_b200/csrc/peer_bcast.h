// Internal layout of b200_bcast (include/b200_gemm.h), shared by the
// exchange protocol (peer_copy.cu) and the GEMM that waits for and releases
// the exchange's slots inside the kernel (b200_gemm.cu).
#pragma once

#include <cuda_runtime.h>

#include "b200_gemm.h"

#include <cstddef>
#include <cstdint>

namespace b200 {
// Receive slots per rank (B200_BCAST_SLOTS): with three, the exchange of
// step s + 2 can run while the GEMM of step s reads its slot, so an exchange
// slower than one GEMM (8 GPUs: ~124 us against ~97) still stays hidden.
constexpr int kBcastSlots = B200_BCAST_SLOTS;
static_assert(kBcastSlots >= 2, "the exchange needs at least two receive slots");
constexpr int kBcastMaxWorld = 8;
// Each piece moves in this many parts, and a receiving rank forwards a part
// as soon as it has landed, so forwarding overlaps rank 0's sending.  With one
// copy stream per peer, 1 and 2 parts gave the same step time on 4 B200s
// (110-113 us) and 1 part the shorter exchange alone (85 against 97 us).
#ifndef B200_BCAST_PARTS
#define B200_BCAST_PARTS 1
#endif
constexpr int kBcastParts = B200_BCAST_PARTS;
}  // namespace b200

struct b200_bcast {
  int rank, world;
  size_t nbytes;
  char* slot[b200::kBcastMaxWorld][b200::kBcastSlots];  // every rank's slots as mapped in this process
  char* flags[b200::kBcastMaxWorld];                    // every rank's flag array as mapped in this process
  // One copy stream per peer this rank writes to (copies to different peers
  // run at the same time on different copy engines), and events to join them
  // with the caller's stream.
  cudaStream_t peer_stream[b200::kBcastMaxWorld];
  cudaEvent_t start_ev;
  cudaEvent_t done_ev[b200::kBcastMaxWorld];
};

namespace b200 {
// Flag array of one rank (uint32): ready[slot][sender][part], done[rank],
// then one counter private to that rank (the in-kernel release's count of
// finished CTA pairs).  A sender's copies into a slot run in order on one
// stream, so ready[slot][sender][last part] means all of them have landed.
inline uint32_t* bcast_ready(const b200_bcast* b, int owner, int slot, int sender, int part) {
  return reinterpret_cast<uint32_t*>(b->flags[owner]) + (slot * b->world + sender) * kBcastParts + part;
}
inline uint32_t* bcast_done(const b200_bcast* b, int owner, int r) {
  return reinterpret_cast<uint32_t*>(b->flags[owner]) + kBcastSlots * b->world * kBcastParts + r;
}
inline uint32_t* bcast_counter(const b200_bcast* b) {
  return reinterpret_cast<uint32_t*>(b->flags[b->rank]) + kBcastSlots * b->world * kBcastParts + b->world;
}
inline size_t bcast_flag_words(int world) { return (size_t)(kBcastSlots * world * kBcastParts + world + 1); }
}  // namespace b200
