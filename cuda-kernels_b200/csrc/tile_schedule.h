// Balanced tile schedule for the CTA-pair GEMM when the output has only a few
// waves of tiles.
//
// With fixed 256 x 512 tiles, a problem whose tile count is not a multiple of
// the number of co-resident CTA pairs leaves pairs idle in the last wave
// (4096^3: 128 tiles on 74 pairs = 1.73 waves, so the kernel takes two full
// tile times while 27 % of the pair-time is idle).  Here the output is cut
// into units of 256 rows x 128 columns instead, numbered row-block by
// row-block; pair p takes the contiguous unit range
// [p*U/P, (p+1)*U/P) of the U units and covers it with tiles of up to four
// units (512 columns) that never cross a row-block.  Every pair then carries
// ceil(U/P) units or one fewer (4096^3: 7 units = 1.75 wide tiles instead of
// 2), and every tile still runs its whole K range in order, so results are
// bit-identical to the fixed tiling.
//
// Plain C++ (host and device): the host picks the schedule, the kernel walks
// it, and a CPU test checks that the tiles cover the output exactly once.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define B200_HD __host__ __device__ __forceinline__
#else
#define B200_HD inline
#endif

namespace b200 {

constexpr int kUnitCols = 128;  // columns per schedule unit
constexpr int kMaxTileUnits = 4;  // 512 columns: the TMEM accumulator

struct BalancedSchedule {
  int32_t units_per_row;  // ceil(N / 128)
  int64_t total_units;    // row blocks x units_per_row
  int32_t pairs;          // CTA pairs sharing the units
};

// Unit range [begin, end) of pair p.
B200_HD void balanced_range(const BalancedSchedule& s, int p, int64_t& begin, int64_t& end) {
  begin = s.total_units * (int64_t)p / s.pairs;
  end = s.total_units * (int64_t)(p + 1) / s.pairs;
}

struct VarTile {
  int32_t mb;     // row block (256 rows)
  int32_t col0;   // first column
  int32_t units;  // width in units of 128 columns (1..4)
};

// Tile starting at unit u of a range ending at `end`: as wide as possible up
// to four units, within the row block.
B200_HD VarTile balanced_tile(const BalancedSchedule& s, int64_t u, int64_t end) {
  VarTile t;
  t.mb = (int32_t)(u / s.units_per_row);
  const int32_t c = (int32_t)(u - (int64_t)t.mb * s.units_per_row);
  int64_t w = s.units_per_row - c;
  if (end - u < w) w = end - u;
  if (w > kMaxTileUnits) w = kMaxTileUnits;
  t.col0 = c * kUnitCols;
  t.units = (int32_t)w;
  return t;
}

}  // namespace b200
