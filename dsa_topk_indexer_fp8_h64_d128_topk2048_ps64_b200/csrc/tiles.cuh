// tiles.cuh — the flat tile sequence the scoring kernels share out.
//
// The 128-token tiles of all scored units (rows, or groups of rows that share
// K pages) are numbered consecutively: unit u owns tiles [start[u],
// start[u+1]) (empty for an unscored unit).  A persistent CTA takes a
// contiguous slice of that sequence and walks it with a Cursor.
#pragma once

namespace dsai {

// Last unit u with start[u] <= t (t < start[units]); that unit is the
// non-empty one holding tile t.
__device__ __forceinline__ int find_row(const int* rs, int rows, int t) {
  int lo = 0, hi = rows - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (rs[mid] <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Walks the tiles of a CTA's slice in order, tracking the unit (`row`) and
// the tile's index inside it (`j`).
struct Cursor {
  int t, row, j, row_end;
  __device__ void init(const int* rs, int rows, int t0) {
    t = t0;
    row = find_row(rs, rows, t0);
    j = t0 - rs[row];
    row_end = rs[row + 1];
  }
  __device__ void next(const int* rs, int t1) {
    ++t;
    ++j;
    if (t < t1 && t == row_end) {
      ++row;
      while (rs[row + 1] <= t) ++row;
      j = 0;
      row_end = rs[row + 1];
    }
  }
};

}  // namespace dsai
