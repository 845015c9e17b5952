// common.cuh — shape contract, row geometry and status reporting shared by
// the indexer kernels.
//
// Shape contract of the operator (reference solution/python/kernel.cu:29-40):
// 64 index heads, head_dim 128, page size 64, top-2048, 8448-B pages made of
// 64x128 e4m3 K values followed by 64 fp32 per-token scales.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/dsai.h"

namespace dsai {

constexpr int kHeads = DSAI_NUM_HEADS;        // 64
constexpr int kDim = DSAI_HEAD_DIM;           // 128 (bytes of e4m3 per token)
constexpr int kPage = DSAI_PAGE_SIZE;         // 64 tokens
constexpr int kTopK = DSAI_TOPK;              // 2048
constexpr int kPageBytes = DSAI_PAGE_BYTES;   // 8448
constexpr int kScaleOff = DSAI_SCALE_OFFSET;  // 8192
constexpr int kPageKBytes = kPage * kDim;     // 8192
constexpr int kTileTok = 128;                 // tokens per UMMA tile (2 pages, M = 128)
constexpr int kQBytes = kHeads * kDim;        // 8192 B of Q per row

// Rows handled by one scoring launch (the per-CTA row table lives in smem);
// the host splits larger batches into several launches.
constexpr int kMaxRowsPerLaunch = 1024;

// First radix digit of the selection: the top 12 bits of the ordered key
// (sign, 8 exponent bits, 3 mantissa bits).  The scorer builds a per-row
// histogram of it in the workspace; the selection kernel consumes it and
// clears it again for the next call.
constexpr int kHistBits = 12;
constexpr int kHistBins = 1 << kHistBits;
// A row's histogram block in the workspace: the 4096 bins, then four u32 of
// per-row counters used by the split selection (output and candidate slots
// taken, chunks finished).  They are zero between calls like the bins.
constexpr int kHistStride = kHistBins + 4;
// Pivot-bin keys the split selection keeps per row (workspace lists).
constexpr int kSplitCap = 4096;

constexpr uint64_t kWaitTimeoutNs = 1000000000ull;  // 1 s bound on any on-chip wait

// Workspace header: status word at offset 0, data from kWsHeader on.
constexpr size_t kWsHeader = 256;
// Control words in the header (int offsets; zero between launches): the
// scorer's next chunk to deal out and its CTAs finished.  (The opt-in fused
// launch keeps its own at ints 16 and 48.)
constexpr int kHdrScoreNext = 24;
constexpr int kHdrScoreDone = 32;

__device__ __forceinline__ void report(int* status, int bits) {
  if (status) atomicOr(status, bits);
}

// Effective length of row b: seq_len clamped to [0, max_pages*64].  Out of
// range values are flagged (the reference would read past the row instead).
__device__ __forceinline__ int row_len(const int32_t* seq_lens, int b, int max_pages,
                                       int* status) {
  const int L = seq_lens[b];
  const int cap = max_pages * kPage;
  const int Lc = L < 0 ? 0 : (L > cap ? cap : L);
  if (Lc != L) report(status, DSAI_STATUS_SEQLEN_CLAMPED);
  return Lc;
}

// Number of 128-token UMMA tiles scored for a row of effective length L.
// Rows that fit entirely in the top-K are not scored (reference early exit,
// solution/python/kernel.cu:102, :576) unless every row is requested.
__device__ __forceinline__ int row_tiles(int L, bool score_all) {
  if (L <= 0) return 0;
  if (L <= kTopK && !score_all) return 0;
  return (L + kTileTok - 1) / kTileTok;
}

// Order-preserving map fp32 -> u32 (larger float -> larger key).  Negative
// values are bit-inverted, non-negative ones get the sign bit set; this is the
// 32-bit form of the reference's HalfToOrderedU16 (kernel.cu:855-859).
__device__ __forceinline__ uint32_t ordered_key(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// Physical slot id of token t of a row (reference kernel.cu:1021-1027).
__device__ __forceinline__ int physical_id(const int32_t* bt_row, int t) {
  return bt_row[t >> 6] * kPage + (t & (kPage - 1));
}

}  // namespace dsai
