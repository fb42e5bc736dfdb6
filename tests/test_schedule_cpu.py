"""CPU check of the balanced tile schedule (cuda-kernels_b200/csrc/tile_schedule.h),
the one the CTA-pair kernel walks for variable-width tiles.

The header is plain C++ on the host; this test compiles it with g++ into a
small program that walks every pair's tile sequence exactly as the kernel's
cursor does and checks, for many shapes and pair counts: every 256 x 128 unit
of the output is covered exactly once, no tile crosses a row block or is
wider than 512 columns, and no pair carries more than ceil(units / pairs)
units."""
import os
import shutil
import subprocess

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CSRC = os.path.join(REPO, "cuda-kernels_b200", "csrc")

PROGRAM = r"""
#include <cstdio>
#include <vector>
#include "tile_schedule.h"
using namespace b200;
int main() {
  const int Ms[] = {1, 200, 256, 257, 4096, 5000, 8191, 8192, 16384};
  const int Ns[] = {1, 100, 128, 129, 1000, 4096, 6144, 28672, 128256};
  const int Ps[] = {1, 2, 37, 73, 74};
  long checked = 0;
  for (int M : Ms) for (int N : Ns) for (int P : Ps) {
    const int mb = (M + 255) / 256;
    BalancedSchedule s{(N + kUnitCols - 1) / kUnitCols, 0, 0};
    s.total_units = (long long)mb * s.units_per_row;
    const int pairs = s.total_units < P ? (int)s.total_units : P;
    s.pairs = pairs;
    std::vector<int> cover((size_t)s.total_units, 0);
    const int64_t cap = (s.total_units + pairs - 1) / pairs;
    for (int p = 0; p < pairs; ++p) {
      int64_t b, e;
      balanced_range(s, p, b, e);
      int64_t u = b, units = 0;
      while (u < e) {
        VarTile t = balanced_tile(s, u, e);
        if (t.units < 1 || t.units > kMaxTileUnits) { printf("bad width %d\n", t.units); return 1; }
        const int c0 = t.col0 / kUnitCols;
        if (t.col0 % kUnitCols || c0 + t.units > s.units_per_row || t.mb >= mb) { printf("tile out of its row block\n"); return 1; }
        for (int i = 0; i < t.units; ++i) cover[(size_t)t.mb * s.units_per_row + c0 + i] += 1;
        units += t.units;
        u += t.units;
      }
      if (units > cap) { printf("pair %d carries %ld > %ld units\n", p, (long)units, (long)cap); return 1; }
    }
    for (int c : cover) if (c != 1) { printf("M=%d N=%d P=%d: a unit covered %d times\n", M, N, P, c); return 1; }
    ++checked;
  }
  printf("ok %ld\n", checked);
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_balanced_schedule_covers_output_exactly_once(tmp_path):
    src = tmp_path / "sched.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "sched"
    subprocess.run(["g++", "-std=c++17", "-O1", "-I", CSRC, str(src), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("ok ")
