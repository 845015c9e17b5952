// radix.cuh — block-level building blocks of the radix top-K selection
// (shared by the selection kernels and the fused score-and-select kernel):
// the warp-aggregated histogram add, warp-collective slot allocation, the
// block-wide search for the bin that holds the k-th largest key, a packed
// block scan, the output writer of a row, and the two-instruction form of the
// order-preserving key map.
#pragma once

#include <cstdint>

#include "common.cuh"

namespace dsai {
namespace radix {

constexpr int kBins2 = 1024;  // 10-bit second and third digits

struct Scan {
  int warp_tot[32];
  int warp_suf[32];
  uint32_t total;
  int sel_bin;
  int sel_above;
  int sel_count;
};

__device__ __forceinline__ void hist_add(uint32_t* hist, uint32_t bin, bool valid) {
  const unsigned active = __ballot_sync(0xffffffffu, valid);
  if (!valid) return;
  const unsigned peers = __match_any_sync(active, bin);
  if ((threadIdx.x & 31) == (__ffs(peers) - 1)) atomicAdd(&hist[bin], __popc(peers));
}

// Warp-collective slot allocation for `cnt` entries of this lane: returns the
// first slot of this lane's entries (one shared atomic per warp).
__device__ __forceinline__ int warp_alloc_n(int* counter, int cnt) {
  const int lane = threadIdx.x & 31;
  int incl = cnt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  const int total = __shfl_sync(0xffffffffu, incl, 31);
  int base = 0;
  if (lane == 31 && total) base = atomicAdd(counter, total);
  base = __shfl_sync(0xffffffffu, base, 31);
  return base + incl - cnt;
}

// The same for a 0/1 flag per lane (a ballot instead of the scan): returns
// this lane's slot, meaningful where flag is set.
__device__ __forceinline__ int warp_alloc_1(int* counter, bool flag) {
  const unsigned m = __ballot_sync(0xffffffffu, flag);
  const int lane = threadIdx.x & 31;
  const int leader = m ? __ffs(m) - 1 : 0;
  int base = 0;
  if (m && lane == leader) base = atomicAdd(counter, __popc(m));
  base = __shfl_sync(0xffffffffu, base, leader);
  return base + __popc(m & ((1u << lane) - 1u));
}

// Finds the bin holding the k-th largest entry of a histogram spread over
// the block (thread t holds bins [t*PER, t*PER + PER) in h): sets sel_bin
// to the bin with above(bin) < k <= above(bin) + count(bin), sel_above to
// above(bin) (entries in higher bins) and sel_count to count(bin); all zero
// if the histogram holds fewer than k entries.  A two-level shuffle suffix
// scan (lanes, then the warp totals, summed by every warp).  Ends with a
// block barrier.
template <int NT, int PER>
__device__ void find_threshold(Scan& sc, const uint32_t (&h)[PER], int k) {
  constexpr int kW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int sum = 0;
#pragma unroll
  for (int i = 0; i < PER; ++i) sum += static_cast<int>(h[i]);
  int v = sum;  // inclusive suffix within the warp (higher lanes own higher bins)
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, v, off);
    if (lane + off < 32) v += y;
  }
  if (lane == 0) sc.warp_tot[warp] = v;
  if (tid == 0) {
    sc.sel_bin = 0;
    sc.sel_above = 0;
    sc.sel_count = 0;
  }
  __syncthreads();
  // Entries in the warps above this one: every warp sums the totals itself
  // (one barrier fewer than a scan by one warp).
  int t = (lane > warp && lane < kW) ? sc.warp_tot[lane] : 0;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) t += __shfl_xor_sync(0xffffffffu, t, off);
  int above = t + (v - sum);
#pragma unroll
  for (int i = PER - 1; i >= 0; --i) {
    const int hi = static_cast<int>(h[i]);
    if (above < k && above + hi >= k) {
      sc.sel_bin = tid * PER + i;
      sc.sel_above = above;
      sc.sel_count = hi;
    }
    above += hi;
  }
  __syncthreads();
}

// Block-wide exclusive scan of a packed pair of counts (low / high 16 bits;
// the totals must stay below 65536).  Returns this thread's exclusive prefix
// and writes the block total to *total.
template <int NT>
__device__ __forceinline__ uint32_t block_scan_packed(Scan& sc, uint32_t v, uint32_t* total) {
  constexpr int kW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) sc.warp_tot[warp] = static_cast<int>(incl);
  __syncthreads();
  if (warp == 0) {
    const uint32_t t = lane < kW ? static_cast<uint32_t>(sc.warp_tot[lane]) : 0u;
    uint32_t ti = t;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, ti, off);
      if (lane >= off) ti += y;
    }
    sc.warp_suf[lane] = static_cast<int>(ti - t);  // exclusive prefix of warp totals
    if (lane == kW - 1) sc.total = ti;
  }
  __syncthreads();
  *total = sc.total;
  return static_cast<uint32_t>(sc.warp_suf[warp]) + incl - v;
}

template <bool kIds>
struct RowOut {
  int32_t* ids;
  float* scores;
  int32_t* tokens;
  int32_t offset;
  // val: the physical id (kIds) or the token index of the entry.  Slots
  // outside the row are dropped: a histogram that disagrees with the logits
  // (a corrupted workspace) can cost the result, never memory safety.
  __device__ __forceinline__ void emit(int pos, int32_t val, uint32_t key) const {
    if (static_cast<unsigned>(pos) >= static_cast<unsigned>(kTopK)) return;
    if constexpr (kIds) {
      ids[pos] = val;
    } else {
      scores[pos] = key_to_float(key);
      tokens[pos] = val + offset;
    }
  }
};

// ordered_key in two integer instructions (arithmetic shift, xor).
__device__ __forceinline__ uint32_t key_of_bits(uint32_t u) {
  return u ^ (static_cast<uint32_t>(static_cast<int32_t>(u) >> 31) | 0x80000000u);
}

}  // namespace radix
}  // namespace dsai
