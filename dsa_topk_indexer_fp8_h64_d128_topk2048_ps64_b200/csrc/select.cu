// select.cu — exact top-2048 selection over fp32 logits, and the merge of
// partial (score, token) candidate lists.
//
// Keys are the order-preserving u32 image of the fp32 logit, so "top-K by
// value" is "top-K by key".  A radix select over three digits (12, 10 and
// 10 key bits) finds the exact 2048-th largest key (the pivot).  The first
// digit's histogram (4096 bins per row) is accumulated by the scoring kernel
// as it writes the logits.
//
// Many rows (select_wide_kernel): one 1024-thread CTA per row.
//   digit 1  thread t reads bins [4t, 4t+4) of the row's histogram and a
//            block suffix scan finds the bin holding the 2048-th largest key
//            (the pivot bin), while the row's first 32768 logits are copied
//            into shared memory;
//   pass     32 entries per thread and round, one mask bit each: keys above
//            the pivot bin go straight to the output, keys in it to a list in
//            shared memory and to the histogram of their next 10 bits; slots
//            come from one shared atomic per warp;
//   refine   the second digit from that histogram; keys above the 22-bit
//            prefix are emitted, and the few keys sharing it (at most 64;
//            else a third digit is counted) are ranked by one warp, which
//            fills the last slots (ties at the pivot in list order).
//
// Few rows (select_split_kernel, described above the kernel): several
// 256-thread CTAs per row, 4096 tokens each, that share the row's output
// slots through atomics on counters in the workspace; the CTA that finishes
// the row last refines it.
//
// Few long rows, the earlier shape kept for comparison (select_rows_kernel,
// used with DSAI_SELECT=rows): one thread-block cluster of C CTAs per row
// (C = 2..8, so that every CTA is resident at once), 256 threads per CTA,
// three CTAs per SM.
//   digit 1  the leader CTA finds the pivot bin and hands it to the
//            cluster's CTAs (distributed shared memory, one cluster barrier)
//            while their first round of logits is copied into shared memory;
//   pass     CTA r classifies its page-aligned segment of the row, 8192
//            entries per round: keys above the pivot bin go straight to the
//            output, at slots taken with one atomic per CTA and round on the
//            leader CTA's counter; keys in the pivot bin are kept, with their
//            output value, in the CTA's own list and counted in its histogram
//            of the next 10 key bits;
//   refine   after a cluster barrier the leader sums the CTAs' histograms to
//            find the second digit, counts the third digit over the lists
//            (read in place through distributed shared memory) and emits the
//            keys above the exact pivot; keys equal to the pivot fill the last
//            slots in arbitrary order.
// If the pivot bin holds more keys than the lists keep (heavily tied
// logits) the refinement runs over the row in global memory instead.  The
// emitted set is exactly a top-K set of the logits; among equal logits at
// the boundary the choice is arbitrary, as in the reference's atomic emit
// (solution/python/kernel.cu:992-1018).
//
// Rows with seq_len <= 2048 emit ids of tokens 0..L-1 in token order and -1
// padding (reference kernel.cu:897-905, :1079-1097).
//
// The merge of (score, token) lists from a page-range split runs the same
// three digits in one 512-thread CTA over the list.
#include <cfloat>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "graph.h"
#include "launch.h"
#include "radix.cuh"
#include "sm100.cuh"

namespace dsai {
namespace {

using sm100::grid_dep_launch_dependents;
using sm100::grid_dep_wait;
using namespace radix;

constexpr int kCandCap = 8192;

// ------------------------------------------------------------ row selection

constexpr int kCPer = 32;        // entries per thread per round (one mask bit each)
constexpr int kCBtCache = 1024;  // block-table entries of a segment in smem
constexpr int kMaxCluster = 8;

// Shape of the cluster kernel (few long rows: C CTAs per row).
template <int NT>
struct SelShape;
template <>
struct SelShape<256> {
  static constexpr int kCtasPerSm = 3;
  static constexpr int kLocalCap = 4096;  // pivot-bin keys one CTA keeps
};

template <int NT>
struct RowSmem {
  static constexpr int kCap = SelShape<NT>::kLocalCap;
  union {
    uint4 hist1[kHistBins / 4];  // staging of the row's first-digit histogram
    struct {
      uint32_t key[kCap];        // this CTA's keys in the pivot bin and their
      int32_t val[kCap];         // output values (physical id or token)
    } cand;
  } u;
  float4 vals[kCPer / 4][NT];    // the current round's logits
  uint32_t hist[kBins2];         // second-digit histogram of this CTA's keys
  int32_t bt[kCBtCache];         // this CTA's pages of the row
  Scan sc;
  const uint32_t* cand_key_of[kMaxCluster];  // leader: every CTA's candidate lists
  const int32_t* cand_val_of[kMaxCluster];
  int gather_base[kMaxCluster + 1];          // leader: prefix of the CTAs' counts
  int bcast[3];                  // the first digit, from the leader: bin, keys above, keys in it
  int out_count;                 // leader: output slots taken (whole row)
  int eq_count;                  // leader: pivot ties taken
  int overflow;                  // leader: some CTA held more than kCap keys
  int cand_count;                // keys this CTA holds
  int base_out;                  // this CTA's first output slot of the current round
};

template <int NT>
constexpr int row_smem_bytes() {
  return static_cast<int>(sizeof(RowSmem<NT>));
}
static_assert(3 * (row_smem_bytes<256>() + 1024) <= 233472, "three 256-thread CTAs per SM must fit");

// Cross-CTA traffic (C > 1) is kept to a few bulk steps: the leader's first
// digit handed to every CTA, one remote atomic per CTA and round (output
// slots), the leader's reads of the other CTAs' counts, histograms and
// candidate lists, and three cluster barriers.  (Per-key remote atomics or
// stores into one CTA's shared memory serialise at that SM and cost
// microseconds.)  With C = 1 the cluster barriers become block barriers.
// Per entry the pass costs a handful of integer instructions; only entries
// above or in the pivot bin are visited again.
template <bool kIds, int NT>
__global__ void __launch_bounds__(NT, SelShape<NT>::kCtasPerSm) select_rows_kernel(const SelectLaunch p) {
  constexpr int kRound = NT * kCPer;
  constexpr int kHistPer = kHistBins / NT;  // first-digit bins per thread
  constexpr int kB2Per = kBins2 / NT;       // refinement bins per thread
  constexpr int kCap = RowSmem<NT>::kCap;
  static_assert(kHistPer % 4 == 0 && kB2Per >= 1, "bin ownership");
  extern __shared__ __align__(16) uint8_t smem_raw[];
  RowSmem<NT>& s = *reinterpret_cast<RowSmem<NT>*>(smem_raw);
  // Launched as a programmatic dependent of the scoring kernel: wait for its
  // logits and histograms, then let the next grid start launching.
  grid_dep_wait();
  grid_dep_launch_dependents();
  const int tid = threadIdx.x;
  const int C = static_cast<int>(sm100::cluster_nctarank());
  const int r = static_cast<int>(sm100::cluster_ctarank());
  const int b = static_cast<int>(sm100::cluster_id_x());
  const int L = row_len(p.seq_lens, b, p.max_pages, nullptr);
  const int32_t* bt_row = p.block_table + static_cast<size_t>(b) * p.max_pages;
  const float* row = p.logits + static_cast<size_t>(b) * p.ld;
  RowOut<kIds> out;
  out.ids = kIds ? p.out_ids + static_cast<size_t>(b) * kTopK : nullptr;
  out.scores = kIds ? nullptr : p.out_scores + static_cast<size_t>(b) * kTopK;
  out.tokens = kIds ? nullptr : p.out_tokens + static_cast<size_t>(b) * kTopK;
  out.offset = p.token_offset;

  if (L <= kTopK) {
    // Every token is selected; the cluster's CTAs share the 2048 slots.  No
    // CTA of this cluster takes a cluster barrier on this path.
    const int i1 = kTopK * (r + 1) / C;
    for (int i = kTopK * r / C + tid; i < i1; i += NT) {
      if constexpr (kIds) {
        out.ids[i] = i < L ? physical_id(bt_row, i) : -1;
      } else {
        out.scores[i] = i < L ? row[i] : -INFINITY;
        out.tokens[i] = i < L ? i + p.token_offset : -1;
      }
    }
    return;
  }

  // Cluster barrier halves (block barriers for a single-CTA cluster).
  auto arrive = [&](bool release) {
    if (C > 1) {
      if (release) sm100::cluster_arrive_release(); else sm100::cluster_arrive_relaxed();
    }
  };
  auto wait = [&]() {
    if (C > 1) sm100::cluster_wait_acquire(); else __syncthreads();
  };

  const bool leader = r == 0;
  // Distributed shared memory is touched only after every CTA of the
  // cluster is known to run (the matching wait).
  arrive(false);
  for (int i = tid; i < kBins2; i += NT) s.hist[i] = 0u;
  if (tid == 0) {
    s.out_count = 0;
    s.eq_count = 0;
    s.overflow = 0;
    s.cand_count = 0;
  }

  // This CTA's segment [s0, s1) of the row: page-aligned, C segments cover it.
  const int seg = ((L + C - 1) / C + kPage - 1) & ~(kPage - 1);
  const int s0 = min(L, r * seg);
  const int s1 = min(L, s0 + seg);
  const float4* row4 = reinterpret_cast<const float4*>(row);
  // One round of logits into shared memory (each thread copies, and later
  // reads, its own 16-B pieces; the row buffer is padded to 64 entries).
  // Pieces at or past s1 are neither read nor copied.
  auto load_round = [&](int base) {
#pragma unroll
    for (int u = 0; u < kCPer / 4; ++u) {
      const int j = base / 4 + u * NT + tid;
      if (4 * j < s1) sm100::cp_async_16(&s.vals[u][tid], row4 + j, 16u);
    }
  };
  if (s0 < s1) load_round(s0);

  const int pg0 = s0 / kPage;
  const int npg = (s1 - s0 + kPage - 1) / kPage;
  const bool bt_cached = kIds && npg <= kCBtCache;
  if (bt_cached)
    for (int i = tid; i < npg; i += NT) s.bt[i] = bt_row[pg0 + i];

  uint32_t* g_hist = p.hist + static_cast<size_t>(b) * kHistStride;
  if (leader) {
    // Digit 1 from the scoring kernel's histogram (cleared below once used):
    // coalesced loads, staged so that each thread owns consecutive bins; the
    // result goes to every CTA of the cluster.
    {
      const uint4* g4 = reinterpret_cast<const uint4*>(g_hist);
      uint4 x[kHistPer / 4];
#pragma unroll
      for (int q = 0; q < kHistPer / 4; ++q) x[q] = g4[q * NT + tid];
#pragma unroll
      for (int q = 0; q < kHistPer / 4; ++q) s.u.hist1[q * NT + tid] = x[q];
    }
    __syncthreads();
    uint32_t h[kHistPer];
#pragma unroll
    for (int q = 0; q < kHistPer / 4; ++q) {
      const uint4 x = s.u.hist1[tid * (kHistPer / 4) + q];
      h[4 * q] = x.x; h[4 * q + 1] = x.y; h[4 * q + 2] = x.z; h[4 * q + 3] = x.w;
    }
    find_threshold<NT, kHistPer>(s.sc, h, kTopK);  // its barriers free the staging area
    wait();
    if (tid < C) {
      int* dst = sm100::cluster_map(s.bcast, static_cast<uint32_t>(tid));
      dst[0] = s.sc.sel_bin;
      dst[1] = s.sc.sel_above;
      dst[2] = s.sc.sel_count;
    }
    uint4* g4 = reinterpret_cast<uint4*>(g_hist);
#pragma unroll
    for (int q = 0; q < kHistPer / 4; ++q) g4[q * NT + tid] = make_uint4(0u, 0u, 0u, 0u);
  } else {
    wait();
  }
  // The first digit and the leader's counters are ready for the cluster.
  arrive(true);
  wait();
  const uint32_t bin1 = static_cast<uint32_t>(s.bcast[0]);
  const int above1 = s.bcast[1];
  const int n1 = s.bcast[2];
  const bool use_cand = n1 <= kCap * C;
  const uint32_t key_lo = bin1 << (32 - kHistBits);                 // first key of the pivot bin
  const uint32_t key_top = key_lo | ((1u << (32 - kHistBits)) - 1u);  // last key of the pivot bin
  int* lead_out = sm100::cluster_map(&s.out_count, 0u);
  int* lead_overflow = sm100::cluster_map(&s.overflow, 0u);

  auto value_of = [&](int i) -> int32_t {
    if constexpr (kIds) {
      const int32_t page = bt_cached ? s.bt[(i >> 6) - pg0] : bt_row[i >> 6];
      return page * kPage + (i & (kPage - 1));
    } else {
      return i;
    }
  };

  for (int base = s0; base < s1; base += kRound) {
    if (base != s0) load_round(base);
    sm100::cp_async_wait_all();  // this thread's own pieces have landed
    // Bit e of gtm / inm: entry e of this thread is above / in-or-above the
    // pivot bin.  Groups of 4 entries wholly past s1 are skipped (uniformly
    // across the block: the groups are NT*4 entries apart).
    uint32_t gtm = 0u, inm = 0u;
    const int groups = min(kCPer / 4, (s1 - base + 4 * NT - 1) / (4 * NT));
#pragma unroll
    for (int u = 0; u < kCPer / 4; ++u) {
      if (u < groups) {
        const uint4 w = *reinterpret_cast<const uint4*>(&s.vals[u][tid]);
        const uint32_t k4[4] = {key_of_bits(w.x), key_of_bits(w.y), key_of_bits(w.z), key_of_bits(w.w)};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (k4[c] > key_top) gtm |= 1u << (4 * u + c);
          if (k4[c] >= key_lo) inm |= 1u << (4 * u + c);
        }
      }
    }
    if (base + kRound > s1) {  // the segment's last round: drop entries at or past s1
      uint32_t valid = 0u;
#pragma unroll
      for (int u = 0; u < kCPer / 4; ++u) {
        const int i0 = base + 4 * (u * NT + tid);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          if (i0 + c < s1) valid |= 1u << (4 * u + c);
      }
      gtm &= valid;
      inm &= valid;
    }
    const uint32_t eqm = use_cand ? (inm & ~gtm) : 0u;
    uint32_t tot;
    const uint32_t pre = block_scan_packed<NT>(s.sc, __popc(gtm) | (__popc(eqm) << 16), &tot);
    const int n_gt = static_cast<int>(tot & 0xFFFFu), n_eq = static_cast<int>(tot >> 16);
    if (tid == 0) s.base_out = n_gt ? atomicAdd(lead_out, n_gt) : 0;
    __syncthreads();
    int pos = s.base_out + static_cast<int>(pre & 0xFFFFu);
    int cpos = s.cand_count + static_cast<int>(pre >> 16);
    uint32_t m = gtm | eqm;
    while (m) {
      const int e = __ffs(m) - 1;
      m &= m - 1u;
      const float x = reinterpret_cast<const float*>(&s.vals[e >> 2][tid])[e & 3];
      const uint32_t key = key_of_bits(__float_as_uint(x));
      const int32_t val = value_of(base + 4 * ((e >> 2) * NT + tid) + (e & 3));
      if ((gtm >> e) & 1u) {
        out.emit(pos++, val, key);
      } else {
        if (cpos < kCap) {
          s.u.cand.key[cpos] = key;
          s.u.cand.val[cpos] = val;
        } else {
          atomicOr(lead_overflow, 1);
        }
        ++cpos;
        atomicAdd(&s.hist[(key >> 10) & (kBins2 - 1)], 1u);
      }
    }
    __syncthreads();  // base_out, cand_count and the scan scratch are reused
    if (tid == 0) s.cand_count += n_eq;
  }
  // Every CTA's candidates, histogram and output slots are final.
  arrive(true);
  wait();

  if (leader) {
    // Counts, list addresses and the summed second-digit histogram of every
    // CTA of the cluster.
    if (tid < 32) {
      int cnt = 0;
      if (tid < C) {
        const uint32_t q = static_cast<uint32_t>(tid);
        cnt = min(*sm100::cluster_map(&s.cand_count, q), kCap);
        s.cand_key_of[tid] = sm100::cluster_map(s.u.cand.key, q);
        s.cand_val_of[tid] = sm100::cluster_map(s.u.cand.val, q);
      }
      int incl = cnt;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, off);
        if (tid >= off) incl += y;
      }
      if (tid < C) s.gather_base[tid] = incl - cnt;
      if (tid == C - 1) s.gather_base[C] = incl;
    }
    uint32_t h2[kB2Per];
#pragma unroll
    for (int i = 0; i < kB2Per; ++i) h2[i] = 0u;
#pragma unroll
    for (int q = 0; q < kMaxCluster; ++q) {
      if (q < C) {
        const uint32_t* src = sm100::cluster_map(&s.hist[tid * kB2Per], static_cast<uint32_t>(q));
        if constexpr (kB2Per == 4) {
          const uint4 x = *reinterpret_cast<const uint4*>(src);
          h2[0] += x.x; h2[1] += x.y; h2[2] += x.z; h2[3] += x.w;
        } else {
#pragma unroll
          for (int i = 0; i < kB2Per; ++i) h2[i] += src[i];
        }
      }
    }
    __syncthreads();  // gather_base, list addresses; every thread has read its own bins

    const bool listed = use_cand && s.overflow == 0;
    const int k1 = kTopK - above1;
    if (!listed) {
      // The pivot bin's keys were not all kept: second digit over the row in
      // global memory instead.
      for (int i = tid; i < kBins2; i += NT) s.hist[i] = 0u;
      __syncthreads();
      for (int base = 0; base < L; base += NT) {
        const int i = base + tid;
        const uint32_t key = i < L ? ordered_key(row[i]) : 0u;
        hist_add(s.hist, (key >> 10) & (kBins2 - 1), i < L && (key >> (32 - kHistBits)) == bin1);
      }
      __syncthreads();
#pragma unroll
      for (int i = 0; i < kB2Per; ++i) h2[i] = s.hist[tid * kB2Per + i];
    }
    find_threshold<NT, kB2Per>(s.sc, h2, k1);
    const uint32_t prefix2 = (bin1 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
    const int k2 = k1 - s.sc.sel_above;

    // Entry j of the pivot bin: from the cluster's lists, or the row.
    const int n3 = listed ? s.gather_base[C] : L;
    auto key_at = [&](int j, int* q_out) -> uint32_t {
      if (!listed) return ordered_key(row[j]);
      int q = 0;
      while (q + 1 < C && j >= s.gather_base[q + 1]) ++q;
      *q_out = q;
      return s.cand_key_of[q][j - s.gather_base[q]];
    };

    // Third digit over the entries that share the 22-bit prefix.
    for (int i = tid; i < kBins2; i += NT) s.hist[i] = 0u;
    __syncthreads();
    for (int base = 0; base < n3; base += NT) {
      const int j = base + tid;
      int q = 0;
      const uint32_t key = j < n3 ? key_at(j, &q) : 0u;
      hist_add(s.hist, key & (kBins2 - 1), j < n3 && (key >> 10) == prefix2);
    }
    __syncthreads();
    uint32_t h3[kB2Per];
#pragma unroll
    for (int i = 0; i < kB2Per; ++i) h3[i] = s.hist[tid * kB2Per + i];
    find_threshold<NT, kB2Per>(s.sc, h3, k2);
    const uint32_t pivot = (prefix2 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
    const int k3 = k2 - s.sc.sel_above;  // how many keys equal to the pivot are taken

    // Emit the pivot bin's keys above the pivot, and k3 keys equal to it.
    for (int base = 0; base < n3; base += NT) {
      const int j = base + tid;
      int q = 0;
      const uint32_t key = j < n3 ? key_at(j, &q) : 0u;
      const bool in_bin = j < n3 && (key >> (32 - kHistBits)) == bin1;
      const bool gt = in_bin && key > pivot;
      const bool eq = in_bin && key == pivot;
      const int pos = warp_alloc_1(&s.out_count, gt);
      const int ticket = warp_alloc_1(&s.eq_count, eq);
      if (gt || (eq && ticket < k3)) {
        int32_t val;
        if (listed) {
          val = s.cand_val_of[q][j - s.gather_base[q]];
        } else if constexpr (kIds) {
          val = physical_id(bt_row, j);
        } else {
          val = j;
        }
        out.emit(gt ? pos : kTopK - k3 + ticket, val, key);
      }
    }
  }
  // The leader has finished reading the other CTAs' shared memory.
  if (C > 1) {
    sm100::cluster_arrive_release();
    sm100::cluster_wait_acquire();
  }
}

// ------------------------------------------------------------ one CTA per row

constexpr int kWThreads = 1024;
constexpr int kWRound = kWThreads * kCPer;  // 32768 entries per round
constexpr int kWCap = 8192;                 // pivot-bin keys kept
constexpr int kWBtCache = 2048;             // block-table entries of a row in smem (131072 tokens)
constexpr int kSmall = 64;                  // second-digit bin small enough for one warp to rank
constexpr int kWideShortRow = 16384;        // rows this short get one wide CTA each, however few

struct WideSmem {
  float4 vals[kCPer / 4][kWThreads];  // the current round's logits
  uint32_t cand_key[kWCap];           // keys in the pivot bin and their output
  int32_t cand_val[kWCap];            // values (physical id or token)
  uint32_t hist[kBins2];              // second (then third) digit histogram
  int32_t bt[kWBtCache];              // the row's pages
  uint32_t small_key[kSmall];         // keys of the second-digit bin
  int32_t small_val[kSmall];
  Scan sc;
  int out_count;
  int cand_count;
  int small_count;
  int eq_count;
  int extreme[3];  // first-digit bins 0 and 4088..4095 (NaN, infinities) are not empty
};

constexpr int kWideSmemBytes = static_cast<int>(sizeof(WideSmem));
static_assert(kWideSmemBytes <= 232448, "the wide CTA must fit");
static_assert(kBins2 == kWThreads && kHistBins == 4 * kWThreads, "bin ownership");
static_assert(kSmall * 16 == kWThreads, "the final ranking uses 16 threads per key");
static_assert(kCPer / 4 == 8, "eight cp.async groups per round");

// One 1024-thread CTA per row: no cross-CTA traffic, and no block-wide scan
// in the pass (output and candidate slots come from one shared atomic per
// warp).  After the pass, the second digit is found from the histogram the
// pass built; the few keys sharing the 22-bit prefix (at most 64, else a
// third digit is counted) are ranked by the block.
template <bool kIds>
__global__ void __launch_bounds__(kWThreads, 1) select_wide_kernel(const SelectLaunch p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  WideSmem& s = *reinterpret_cast<WideSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int b = blockIdx.x;
  // Before the wait on the scoring kernel: what does not depend on it.  This
  // kernel's predecessor in the stream is that scoring launch, which writes
  // neither seq_lens nor the block table, and started its own work only after
  // its predecessors had completed.
  const int L = row_len(p.seq_lens, b, p.max_pages, nullptr);
  const int32_t* bt_row = p.block_table + static_cast<size_t>(b) * p.max_pages;
  const float* row = p.logits + static_cast<size_t>(b) * p.ld;
  RowOut<kIds> out;
  out.ids = kIds ? p.out_ids + static_cast<size_t>(b) * kTopK : nullptr;
  out.scores = kIds ? nullptr : p.out_scores + static_cast<size_t>(b) * kTopK;
  out.tokens = kIds ? nullptr : p.out_tokens + static_cast<size_t>(b) * kTopK;
  out.offset = p.token_offset;

  if (L <= kTopK) {  // every token is selected
    if constexpr (!kIds) grid_dep_wait();  // the pairs carry the scores
    for (int i = tid; i < kTopK; i += kWThreads) {
      if constexpr (kIds) {
        out.ids[i] = i < L ? physical_id(bt_row, i) : -1;
      } else {
        out.scores[i] = i < L ? row[i] : -INFINITY;
        out.tokens[i] = i < L ? i + p.token_offset : -1;
      }
    }
    // Every CTA waits before it ends, so that this grid completes only after
    // the scoring grid (the next launch's wait relies on it).
    if constexpr (kIds) grid_dep_wait();
    grid_dep_launch_dependents();
    return;
  }
  if (tid == 0) {
    s.out_count = 0;
    s.cand_count = 0;
    s.small_count = 0;
    s.eq_count = 0;
  }
  const int npg = (L + kPage - 1) / kPage;
  const bool bt_cached = kIds && npg <= kWBtCache;
  if (bt_cached)
    for (int i = tid; i < npg; i += kWThreads) s.bt[i] = bt_row[i];
  s.hist[tid] = 0u;

  // The scoring kernel's logits and histograms are complete past this wait.
  grid_dep_wait();
  grid_dep_launch_dependents();
  // Digit 1: thread t owns bins [4t, 4t + 4) of the scoring kernel's
  // histogram (one coalesced 16-B load), cleared for the next call once read.
  uint4* g4 = reinterpret_cast<uint4*>(p.hist + static_cast<size_t>(b) * kHistStride);
  const uint4 hx = g4[tid];

  // A round of logits into shared memory: every thread copies its own 16 B
  // of each group of 4 * kWThreads entries (one cp.async group per group of
  // entries) and reads only those slots, so it waits for its own copies
  // (cp.async.wait_group) and the classification of a group starts as soon
  // as it has landed.  The row buffer is padded to 64 entries, so a float4
  // that starts below the row's end stays inside it; past the end the copy
  // zero-fills without reading.
  auto load_round = [&](int base) {
    const int n = min(L - base, kWRound);
#pragma unroll
    for (int u = 0; u < kCPer / 4; ++u) {
      const int e = u * 4 * kWThreads + 4 * tid;
      sm100::cp_async_16(&s.vals[u][tid], e < n ? row + base + e : row, e < n ? 16u : 0u);
      sm100::cp_async_commit_group();
    }
  };
  load_round(0);

  uint32_t h1[4] = {hx.x, hx.y, hx.z, hx.w};
  if (tid == 0) s.extreme[0] = h1[0] != 0u;
  if (tid >= kWThreads - 2) s.extreme[tid - (kWThreads - 3)] = (h1[0] | h1[1] | h1[2] | h1[3]) != 0u;
  find_threshold<kWThreads, 4>(s.sc, h1, kTopK);  // its barriers publish the zeroed counters
  g4[tid] = make_uint4(0u, 0u, 0u, 0u);
  const uint32_t bin1 = static_cast<uint32_t>(s.sc.sel_bin);
  const int above1 = s.sc.sel_above;
  const int n1 = s.sc.sel_count;
  const bool listed = n1 <= kWCap;
  const uint32_t key_lo = bin1 << (32 - kHistBits);
  const uint32_t key_top = key_lo | ((1u << (32 - kHistBits)) - 1u);
  const int k1 = kTopK - above1;
  // A group of 4 logits whose float maximum is below the pivot bin's first
  // value holds no key in or above the bin and is skipped after 4 compares.
  // Exact for every non-NaN value (the key order is the float order, and a
  // bound of +0.0 never skips -0.0); rows whose histogram shows NaNs or
  // infinities (bins 0 and 4088..4095) classify every entry by its key.
  const bool fast_skip = (s.extreme[0] | s.extreme[1] | s.extreme[2]) == 0;
  const float f_lo = key_to_float(key_lo);

  auto value_of = [&](int i) -> int32_t {
    if constexpr (kIds) {
      const int32_t page = bt_cached ? s.bt[i >> 6] : bt_row[i >> 6];
      return page * kPage + (i & (kPage - 1));
    } else {
      return i;
    }
  };

  for (int base = 0; base < L; base += kWRound) {
    if (base != 0) load_round(base);  // each thread refills only its own slots
    uint32_t gtm = 0u, inm = 0u;
    // Groups u < groups hold entries below L; only the last one can be
    // partial (entries of group u end at base + 4 * (u + 1) * kWThreads).
    const int groups = min(kCPer / 4, (L - base + 4 * kWThreads - 1) / (4 * kWThreads));
#pragma unroll
    for (int u = 0; u < kCPer / 4; ++u) {
      if (u < groups) {
        switch (u) {  // this thread's copies of groups 0..u have landed
          case 0: sm100::cp_async_wait_group<7>(); break;
          case 1: sm100::cp_async_wait_group<6>(); break;
          case 2: sm100::cp_async_wait_group<5>(); break;
          case 3: sm100::cp_async_wait_group<4>(); break;
          case 4: sm100::cp_async_wait_group<3>(); break;
          case 5: sm100::cp_async_wait_group<2>(); break;
          case 6: sm100::cp_async_wait_group<1>(); break;
          default: sm100::cp_async_wait_group<0>(); break;
        }
        const float4 w = s.vals[u][tid];
        if (fast_skip && fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)) < f_lo) continue;
        const uint32_t k4[4] = {key_of_bits(__float_as_uint(w.x)), key_of_bits(__float_as_uint(w.y)),
                                key_of_bits(__float_as_uint(w.z)), key_of_bits(__float_as_uint(w.w))};
        uint32_t g = 0u, n = 0u;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          g |= static_cast<uint32_t>(k4[c] > key_top) << c;
          n |= static_cast<uint32_t>(k4[c] >= key_lo) << c;
        }
        if (u == groups - 1) {  // entries at or past L
          const int left = L - (base + 4 * (u * kWThreads + tid));
          const uint32_t valid = left >= 4 ? 0xFu : (left > 0 ? (1u << left) - 1u : 0u);
          g &= valid;
          n &= valid;
        }
        gtm |= g << (4 * u);
        inm |= n << (4 * u);
      }
    }
    const uint32_t eqm = listed ? (inm & ~gtm) : 0u;
    int pos = warp_alloc_n(&s.out_count, __popc(gtm));
    int cpos = warp_alloc_n(&s.cand_count, __popc(eqm));
    auto entry = [&](int e) { return base + 4 * ((e >> 2) * kWThreads + tid) + (e & 3); };
    auto key_of_entry = [&](int e) {
      return key_of_bits(__float_as_uint(reinterpret_cast<const float*>(&s.vals[e >> 2][tid])[e & 3]));
    };
    for (uint32_t m = gtm; m; m &= m - 1u) {  // above the pivot bin: straight to the output
      const int e = __ffs(m) - 1;
      out.emit(pos++, value_of(entry(e)), kIds ? 0u : key_of_entry(e));
    }
    for (uint32_t m = eqm; m; m &= m - 1u) {  // in the pivot bin: to the list
      const int e = __ffs(m) - 1;
      const uint32_t key = key_of_entry(e);
      if (cpos < kWCap) {
        s.cand_key[cpos] = key;
        s.cand_val[cpos] = value_of(entry(e));
      }
      ++cpos;
      atomicAdd(&s.hist[(key >> 10) & (kBins2 - 1)], 1u);
    }
  }
  sm100::cp_async_wait_group<0>();  // groups past the row's end (zero-fills) too
  __syncthreads();  // candidates, second-digit counts and output slots are final

  if (!listed) {
    // More keys in the pivot bin than the list holds: the second digit over
    // the row in global memory.
    for (int base = 0; base < L; base += kWThreads) {
      const int i = base + tid;
      const uint32_t key = i < L ? ordered_key(row[i]) : 0u;
      hist_add(s.hist, (key >> 10) & (kBins2 - 1), i < L && (key >> (32 - kHistBits)) == bin1);
    }
    __syncthreads();
  }
  uint32_t h2[1] = {s.hist[tid]};
  find_threshold<kWThreads, 1>(s.sc, h2, k1);
  const uint32_t prefix2 = (bin1 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
  const int k2 = k1 - s.sc.sel_above;  // keys still needed from the second-digit bin
  const int n2 = s.sc.sel_count;
  const bool small = n2 <= kSmall;

  // The pivot bin's entries: the list, or the row.
  const int n3 = listed ? min(s.cand_count, kWCap) : L;
  auto key_at = [&](int j) -> uint32_t {
    if (listed) return s.cand_key[j];
    const uint32_t key = ordered_key(row[j]);
    return (key >> (32 - kHistBits)) == bin1 ? key : 0u;
  };
  auto val_at = [&](int j) -> int32_t {
    if (listed) return s.cand_val[j];
    if constexpr (kIds) return physical_id(bt_row, j); else return j;
  };

  if (small) {
    // Emit the keys above the 22-bit prefix; collect the prefix's keys.
    for (int base = 0; base < n3; base += kWThreads) {
      const int j = base + tid;
      const uint32_t key = j < n3 ? key_at(j) : 0u;
      const bool in = j < n3 && key != 0u && (key >> (32 - kHistBits)) == bin1;
      const bool gt = in && (key >> 10) > prefix2;
      const bool eq = in && (key >> 10) == prefix2;
      const int pos = warp_alloc_1(&s.out_count, gt);
      const int q = warp_alloc_1(&s.small_count, eq);
      if (gt) out.emit(pos, val_at(j), key);
      if (eq && q < kSmall) {
        s.small_key[q] = key;
        s.small_val[q] = val_at(j);
      }
    }
    __syncthreads();
    {
      // Rank the n2 keys (largest first, ties by list position) with the
      // whole block: key i is compared with keys 4c..4c+3 by thread 16i + c
      // and the 16 partial counts are summed over those lanes (one step of
      // latency instead of a 32-step chain in one warp).  The k2 best take
      // the last k2 slots.
      const int n = min(s.small_count, kSmall);
      const int i = tid >> 4, c = tid & 15;
      const uint32_t ki = i < n ? s.small_key[i] : 0u;
      int r = 0;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int j = 4 * c + q;
        const uint32_t kj = j < n ? s.small_key[j] : 0u;
        r += (j < n && (kj > ki || (kj == ki && j < i))) ? 1 : 0;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
      if (c == 0 && i < n && r < k2) out.emit(kTopK - k2 + r, s.small_val[i], ki);
    }
    return;
  }

  // Many keys share the 22-bit prefix: count the third digit over them.
  s.hist[tid] = 0u;
  __syncthreads();
  for (int base = 0; base < n3; base += kWThreads) {
    const int j = base + tid;
    const uint32_t key = j < n3 ? key_at(j) : 0u;
    if (j < n3 && key != 0u && (key >> 10) == prefix2) atomicAdd(&s.hist[key & (kBins2 - 1)], 1u);
  }
  __syncthreads();
  uint32_t h3[1] = {s.hist[tid]};
  find_threshold<kWThreads, 1>(s.sc, h3, k2);
  const uint32_t pivot = (prefix2 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
  const int k3 = k2 - s.sc.sel_above;  // how many keys equal to the pivot are taken
  for (int base = 0; base < n3; base += kWThreads) {
    const int j = base + tid;
    const uint32_t key = j < n3 ? key_at(j) : 0u;
    const bool in = j < n3 && key != 0u && (key >> (32 - kHistBits)) == bin1;
    const bool gt = in && key > pivot;
    const bool eq = in && key == pivot;
    const int pos = warp_alloc_1(&s.out_count, gt);
    const int ticket = warp_alloc_1(&s.eq_count, eq);
    if (gt) out.emit(pos, val_at(j), key);
    if (eq && ticket < k3) out.emit(kTopK - k3 + ticket, val_at(j), key);
  }
}

// ------------------------------------------------------------ several CTAs per row

// Split selection: CTA (b, c) of a grid of rows x chunks_per_row handles
// tokens [4096c, 4096c + 4096) of row b; CTAs past the row's end leave at
// once.  Every CTA of a row finds the same pivot bin from the row's
// histogram, classifies its chunk, takes output and list slots with one
// 64-bit atomic on the row's counters, emits the keys above the pivot bin
// and appends the keys in it to the row's list in the workspace.  The CTA
// that finishes last (a ticket counter) refines over that list: the second
// digit, then the <= 64 keys sharing the 22-bit prefix ranked by the block
// (or a third digit); it also clears the row's histogram and counters for
// the next call.  No CTA waits for another: the last one only reads what the
// others published before they took their tickets.  A long row is thus
// streamed by many SMs at once instead of one (one SM pulls ~50 GB/s of
// logits from L2).
constexpr int kSThreads = 256;
constexpr int kSPer = 16;                   // entries per thread
constexpr int kSChunk = kSThreads * kSPer;  // 4096 tokens per CTA
constexpr int kSSmall = 64;                 // second-digit bin small enough to rank directly
constexpr int kSStage = kSChunk / 2;        // list entries the last CTA stages in shared memory

// The row's counters, stored after its 4096 histogram bins (zero between
// calls).
struct RowCtl {
  unsigned long long slots;  // output slots (low 32 bits) and list slots (high 32 bits) taken
  unsigned int done;         // CTAs of the row finished
  unsigned int pad;
};
static_assert(sizeof(RowCtl) == (kHistStride - kHistBins) * sizeof(uint32_t), "counter block");

struct SplitSmem {
  union {
    float4 vals[kSPer / 4][kSThreads];  // the chunk's logits
    struct {
      uint32_t key[kSStage];            // last CTA: the first entries of the row's
      int32_t val[kSStage];             // pivot-bin list (the rest stays in L2)
    } list;
  } u;
  uint32_t hist[kBins2];                // second (then third) digit histogram
  int32_t bt[kSChunk / kPage];          // the chunk's pages
  uint32_t small_key[kSSmall];
  int32_t small_val[kSSmall];
  Scan sc;
  int extreme[2];  // first-digit bins 0 and 4088..4095 (NaN, infinities) are not empty
  int base_out;
  int base_cand;
  int last;
  int out_count;
  int n_cand;
  int small_count;
  int eq_count;
};

constexpr int kSplitSmemBytes = static_cast<int>(sizeof(SplitSmem));
static_assert(sizeof(SplitSmem::u) == kSPer / 4 * kSThreads * 16, "the list staging reuses the logits buffer");
static_assert(kSStage % kSThreads == 0, "list staging");
static_assert(kSplitCap / kSThreads <= 32, "a 32-bit mask of list entries per thread");
static_assert(kSThreads == 4 * kSSmall, "four threads rank each of the 64 keys");

template <bool kIds>
__global__ void __launch_bounds__(kSThreads, 4) select_split_kernel(const SelectLaunch p, int chunks_per_row) {
  constexpr int kHPer = kHistBins / kSThreads;  // 16 first-digit bins per thread
  constexpr int kB2Per = kBins2 / kSThreads;    // 4 refinement bins per thread
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SplitSmem& s = *reinterpret_cast<SplitSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int b = static_cast<int>(blockIdx.x) / chunks_per_row;
  const int c = static_cast<int>(blockIdx.x) - b * chunks_per_row;
  // Before the wait on the scoring kernel: seq_lens and the block table,
  // which it does not write.
  const int L = row_len(p.seq_lens, b, p.max_pages, nullptr);
  const int nch = L > kTopK ? (L + kSChunk - 1) / kSChunk : 1;
  if (c >= nch) return;  // CTA (b, 0) exists for every row, and it waits
  const int32_t* bt_row = p.block_table + static_cast<size_t>(b) * p.max_pages;
  const float* row = p.logits + static_cast<size_t>(b) * p.ld;
  RowOut<kIds> out;
  out.ids = kIds ? p.out_ids + static_cast<size_t>(b) * kTopK : nullptr;
  out.scores = kIds ? nullptr : p.out_scores + static_cast<size_t>(b) * kTopK;
  out.tokens = kIds ? nullptr : p.out_tokens + static_cast<size_t>(b) * kTopK;
  out.offset = p.token_offset;

  if (L <= kTopK) {  // every token is selected
    if constexpr (!kIds) grid_dep_wait();  // the pairs carry the scores
    for (int i = tid; i < kTopK; i += kSThreads) {
      if constexpr (kIds) {
        out.ids[i] = i < L ? physical_id(bt_row, i) : -1;
      } else {
        out.scores[i] = i < L ? row[i] : -INFINITY;
        out.tokens[i] = i < L ? i + p.token_offset : -1;
      }
    }
    if constexpr (kIds) grid_dep_wait();  // the grid completes after the scoring grid
    grid_dep_launch_dependents();
    return;
  }
  const int t0 = c * kSChunk;
  const int t1 = min(L, t0 + kSChunk);
  const int pg0 = t0 / kPage;
  if constexpr (kIds) {
    const int npg = (t1 - t0 + kPage - 1) / kPage;
    for (int i = tid; i < npg; i += kSThreads) s.bt[i] = bt_row[pg0 + i];
  }
  uint32_t* g_hist = p.hist + static_cast<size_t>(b) * kHistStride;
  RowCtl* ctl = reinterpret_cast<RowCtl*>(g_hist + kHistBins);
  uint32_t* list_key = p.cand + static_cast<size_t>(b) * (2 * kSplitCap);
  int32_t* list_val = reinterpret_cast<int32_t*>(list_key + kSplitCap);

  // The scoring kernel's logits and histograms are complete past this wait.
  grid_dep_wait();
  grid_dep_launch_dependents();
  // Digit 1: thread t owns bins [16t, 16t + 16) of the row's histogram.
  // These loads go out before the logits' copies, which would otherwise
  // queue ahead of them.
  uint32_t h[kHPer];
  {
    const uint4* g4 = reinterpret_cast<const uint4*>(g_hist) + tid * (kHPer / 4);
    uint4 x[kHPer / 4];
#pragma unroll
    for (int q = 0; q < kHPer / 4; ++q) x[q] = __ldcg(g4 + q);
#pragma unroll
    for (int q = 0; q < kHPer / 4; ++q) {
      h[4 * q] = x[q].x; h[4 * q + 1] = x[q].y; h[4 * q + 2] = x[q].z; h[4 * q + 3] = x[q].w;
    }
  }
  // The chunk's logits: every thread copies (and later reads) its own 16 B
  // of each group of 4 * kSThreads entries, one cp.async group per group.
  // The row buffer is padded to 64 entries, so a float4 that starts below
  // the row's end stays inside it; past the end the copy zero-fills.
#pragma unroll
  for (int u = 0; u < kSPer / 4; ++u) {
    const int i = t0 + u * 4 * kSThreads + 4 * tid;
    sm100::cp_async_16(&s.u.vals[u][tid], i < t1 ? row + i : row, i < t1 ? 16u : 0u);
    sm100::cp_async_commit_group();
  }
  if (tid == 0) s.extreme[0] = h[0] != 0u;
  if (tid == kSThreads - 1) {
    uint32_t e = 0u;
#pragma unroll
    for (int i = kHPer - 8; i < kHPer; ++i) e |= h[i];
    s.extreme[1] = e != 0u;
  }
  find_threshold<kSThreads, kHPer>(s.sc, h, kTopK);  // ends with a barrier
  const uint32_t bin1 = static_cast<uint32_t>(s.sc.sel_bin);
  const int above1 = s.sc.sel_above;
  const int n1 = s.sc.sel_count;
  const bool listed = n1 <= kSplitCap;
  const uint32_t key_lo = bin1 << (32 - kHistBits);
  const uint32_t key_top = key_lo | ((1u << (32 - kHistBits)) - 1u);
  // A group of 4 logits whose float maximum is below the pivot bin's first
  // value is skipped after 4 compares (exact for non-NaN values; rows whose
  // histogram shows NaNs or infinities classify every entry by its key).
  const bool fast_skip = (s.extreme[0] | s.extreme[1]) == 0;
  const float f_lo = key_to_float(key_lo);

  uint32_t gtm = 0u, inm = 0u;
#pragma unroll
  for (int u = 0; u < kSPer / 4; ++u) {
    switch (u) {  // this thread's copies of groups 0..u have landed
      case 0: sm100::cp_async_wait_group<3>(); break;
      case 1: sm100::cp_async_wait_group<2>(); break;
      case 2: sm100::cp_async_wait_group<1>(); break;
      default: sm100::cp_async_wait_group<0>(); break;
    }
    const int i0 = t0 + u * 4 * kSThreads + 4 * tid;
    if (i0 >= t1) continue;
    const float4 w = s.u.vals[u][tid];
    if (fast_skip && fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)) < f_lo) continue;
    const uint32_t k4[4] = {key_of_bits(__float_as_uint(w.x)), key_of_bits(__float_as_uint(w.y)),
                            key_of_bits(__float_as_uint(w.z)), key_of_bits(__float_as_uint(w.w))};
    uint32_t g = 0u, n = 0u;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      g |= static_cast<uint32_t>(k4[q] > key_top) << q;
      n |= static_cast<uint32_t>(k4[q] >= key_lo) << q;
    }
    const int left = t1 - i0;
    if (left < 4) {  // entries at or past the row's end
      const uint32_t valid = (1u << left) - 1u;
      g &= valid;
      n &= valid;
    }
    gtm |= g << (4 * u);
    inm |= n << (4 * u);
  }
  const uint32_t eqm = listed ? (inm & ~gtm) : 0u;

  // Output and list slots of the chunk: one atomic on the row's counters.
  uint32_t tot;
  const uint32_t pre = block_scan_packed<kSThreads>(s.sc, __popc(gtm) | (__popc(eqm) << 16), &tot);
  if (tid == 0) {
    const unsigned long long add =
        (tot & 0xFFFFu) | (static_cast<unsigned long long>(tot >> 16) << 32);
    const unsigned long long old = add ? atomicAdd(&ctl->slots, add) : 0ull;
    s.base_out = static_cast<int>(old & 0xFFFFFFFFull);
    s.base_cand = static_cast<int>(old >> 32);
  }
  __syncthreads();
  auto value_of = [&](int i) -> int32_t {
    if constexpr (kIds) {
      return s.bt[(i >> 6) - pg0] * kPage + (i & (kPage - 1));
    } else {
      return i;
    }
  };
  {
    int pos = s.base_out + static_cast<int>(pre & 0xFFFFu);
    int cpos = s.base_cand + static_cast<int>(pre >> 16);
    auto entry = [&](int e) { return t0 + (e >> 2) * 4 * kSThreads + 4 * tid + (e & 3); };
    auto key_of_entry = [&](int e) {
      return key_of_bits(__float_as_uint(reinterpret_cast<const float*>(&s.u.vals[e >> 2][tid])[e & 3]));
    };
    for (uint32_t m = gtm; m; m &= m - 1u) {  // above the pivot bin: straight to the output
      const int e = __ffs(m) - 1;
      out.emit(pos++, value_of(entry(e)), kIds ? 0u : key_of_entry(e));
    }
    for (uint32_t m = eqm; m; m &= m - 1u) {  // in the pivot bin: to the row's list
      const int e = __ffs(m) - 1;
      if (cpos < kSplitCap) {
        list_key[cpos] = key_of_entry(e);
        list_val[cpos] = value_of(entry(e));
      }
      ++cpos;
    }
  }

  // Ticket: the CTA that finishes the row last refines it.  The barrier and
  // thread 0's fence order the block's output and list writes before its
  // ticket; the last CTA's fence after the final ticket makes every other
  // CTA's writes visible to its loads.
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned int t = atomicAdd(&ctl->done, 1u);
    const int last = t == static_cast<unsigned int>(nch - 1);
    if (last) __threadfence();
    s.last = last;
  }
  __syncthreads();
  if (!s.last) return;

  // The first kSStage list entries are loaded at once, before their count
  // is known (one round trip; entries past the count are ignored).
  constexpr int kStPer = kSStage / kSThreads;
  uint32_t st_key[kStPer];
  int32_t st_val[kStPer];
  if (listed) {
#pragma unroll
    for (int q = 0; q < kStPer; ++q) {
      st_key[q] = __ldcg(list_key + q * kSThreads + tid);
      st_val[q] = __ldcg(list_val + q * kSThreads + tid);
    }
  }
  if (tid == 0) {
    const unsigned long long v = __ldcg(&ctl->slots);
    s.out_count = static_cast<int>(v & 0xFFFFFFFFull);
    s.n_cand = static_cast<int>(v >> 32);
    s.small_count = 0;
    s.eq_count = 0;
    ctl->slots = 0ull;  // every CTA of the row has taken its slots and ticket
    ctl->done = 0u;
  }
  {
    // Every CTA of the row has read the histogram: clear it for the next call.
    uint4* g4 = reinterpret_cast<uint4*>(g_hist) + tid * (kHPer / 4);
#pragma unroll
    for (int q = 0; q < kHPer / 4; ++q) g4[q] = make_uint4(0u, 0u, 0u, 0u);
  }
  for (int i = tid; i < kBins2; i += kSThreads) s.hist[i] = 0u;
  if (listed) {
#pragma unroll
    for (int q = 0; q < kStPer; ++q) {
      s.u.list.key[q * kSThreads + tid] = st_key[q];
      s.u.list.val[q * kSThreads + tid] = st_val[q];
    }
  }
  __syncthreads();
  const int n3 = listed ? min(s.n_cand, kSplitCap) : L;
  // Entry j of the pivot bin: from the list (its first kSStage entries
  // staged in shared memory), or (more keys in the bin than the list keeps)
  // from the row in global memory, 0 if not in the bin.
  auto key_at = [&](int j) -> uint32_t {
    if (listed) return j < kSStage ? s.u.list.key[j] : __ldcg(list_key + j);
    const uint32_t key = ordered_key(__ldcg(row + j));
    return (key >> (32 - kHistBits)) == bin1 ? key : 0u;
  };
  auto val_at = [&](int j) -> int32_t {
    if (listed) return j < kSStage ? s.u.list.val[j] : __ldcg(list_val + j);
    if constexpr (kIds) return physical_id(bt_row, j); else return j;
  };

  for (int base = 0; base < n3; base += kSThreads) {
    const int j = base + tid;
    const uint32_t key = j < n3 ? key_at(j) : 0u;
    if (j < n3 && key != 0u && (key >> (32 - kHistBits)) == bin1) atomicAdd(&s.hist[(key >> 10) & (kBins2 - 1)], 1u);
  }
  __syncthreads();
  uint32_t h2[kB2Per];
#pragma unroll
  for (int i = 0; i < kB2Per; ++i) h2[i] = s.hist[tid * kB2Per + i];
  const int k1 = kTopK - above1;
  find_threshold<kSThreads, kB2Per>(s.sc, h2, k1);
  const uint32_t prefix2 = (bin1 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
  const int k2 = k1 - s.sc.sel_above;  // keys still needed from the second-digit bin
  const int n2 = s.sc.sel_count;

  if (n2 <= kSSmall) {
    // Emit the keys above the 22-bit prefix; collect the prefix's keys.
    if (listed) {
      // Every thread classifies all its list entries (j = tid + 256q) first,
      // then takes its output and small-list slots with one allocation each
      // (not one pair per 256 entries).
      constexpr int kLPer = kSplitCap / kSThreads;
      uint32_t gtb = 0u, eqb = 0u;
#pragma unroll
      for (int q = 0; q < kLPer; ++q) {
        const int j = q * kSThreads + tid;
        const uint32_t key = j < n3 ? key_at(j) : 0u;
        const bool in = key != 0u && (key >> (32 - kHistBits)) == bin1;
        gtb |= static_cast<uint32_t>(in && (key >> 10) > prefix2) << q;
        eqb |= static_cast<uint32_t>(in && (key >> 10) == prefix2) << q;
      }
      int pos = warp_alloc_n(&s.out_count, __popc(gtb));
      int qs = warp_alloc_n(&s.small_count, __popc(eqb));
      for (uint32_t m = gtb; m; m &= m - 1u) {
        const int j = (__ffs(m) - 1) * kSThreads + tid;
        out.emit(pos++, val_at(j), key_at(j));
      }
      for (uint32_t m = eqb; m; m &= m - 1u, ++qs) {
        const int j = (__ffs(m) - 1) * kSThreads + tid;
        if (qs < kSSmall) {
          s.small_key[qs] = key_at(j);
          s.small_val[qs] = val_at(j);
        }
      }
    } else {
      for (int base = 0; base < n3; base += kSThreads) {
        const int j = base + tid;
        const uint32_t key = j < n3 ? key_at(j) : 0u;
        const bool in = j < n3 && key != 0u && (key >> (32 - kHistBits)) == bin1;
        const bool gt = in && (key >> 10) > prefix2;
        const bool eq = in && (key >> 10) == prefix2;
        const int pos = warp_alloc_1(&s.out_count, gt);
        const int q = warp_alloc_1(&s.small_count, eq);
        if (gt) out.emit(pos, val_at(j), key);
        if (eq && q < kSSmall) {
          s.small_key[q] = key;
          s.small_val[q] = val_at(j);
        }
      }
    }
    __syncthreads();
    // Rank the n2 keys (largest first, ties by list position): key i is
    // compared with keys 16c..16c+15 by thread 4i + c and the four partial
    // counts are summed; the k2 best take the last k2 slots.
    const int n = min(s.small_count, kSSmall);
    const int i = tid >> 2, c4 = tid & 3;
    const uint32_t ki = i < n ? s.small_key[i] : 0u;
    int r = 0;
#pragma unroll
    for (int q = 0; q < kSSmall / 4; ++q) {
      const int j = (kSSmall / 4) * c4 + q;
      const uint32_t kj = j < n ? s.small_key[j] : 0u;
      r += (j < n && (kj > ki || (kj == ki && j < i))) ? 1 : 0;
    }
    r += __shfl_xor_sync(0xffffffffu, r, 2);
    r += __shfl_xor_sync(0xffffffffu, r, 1);
    if (c4 == 0 && i < n && r < k2) out.emit(kTopK - k2 + r, s.small_val[i], ki);
    return;
  }

  // Many keys share the 22-bit prefix: count the third digit over them.
  for (int i = tid; i < kBins2; i += kSThreads) s.hist[i] = 0u;
  __syncthreads();
  for (int base = 0; base < n3; base += kSThreads) {
    const int j = base + tid;
    const uint32_t key = j < n3 ? key_at(j) : 0u;
    if (j < n3 && key != 0u && (key >> 10) == prefix2) atomicAdd(&s.hist[key & (kBins2 - 1)], 1u);
  }
  __syncthreads();
  uint32_t h3[kB2Per];
#pragma unroll
  for (int i = 0; i < kB2Per; ++i) h3[i] = s.hist[tid * kB2Per + i];
  find_threshold<kSThreads, kB2Per>(s.sc, h3, k2);
  const uint32_t pivot = (prefix2 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
  const int k3 = k2 - s.sc.sel_above;  // how many keys equal to the pivot are taken
  for (int base = 0; base < n3; base += kSThreads) {
    const int j = base + tid;
    const uint32_t key = j < n3 ? key_at(j) : 0u;
    const bool in = j < n3 && key != 0u && (key >> (32 - kHistBits)) == bin1;
    const bool gt = in && key > pivot;
    const bool eq = in && key == pivot;
    const int pos = warp_alloc_1(&s.out_count, gt);
    const int ticket = warp_alloc_1(&s.eq_count, eq);
    if (gt) out.emit(pos, val_at(j), key);
    if (eq && ticket < k3) out.emit(kTopK - k3 + ticket, val_at(j), key);
  }
}

// ------------------------------------------------------------ merge

constexpr int kMThreads = 512;
constexpr int kMergeStage = 16384;  // candidate keys staged in shared memory (8 ranks' lists)

struct MergeSmem {
  uint32_t key_all[kMergeStage];
  uint32_t hist[kHistBins];
  uint32_t cand_key[kCandCap];
  int32_t cand_idx[kCandCap];
  Scan sc;
  int out_count;
  int cand_count;
  int eq_count;
};

constexpr int kMergeSmemBytes = static_cast<int>(sizeof(MergeSmem));

// Key of candidate i of a (score, token) list; padding (token -1) and tokens
// >= L are no entry (key 0, never produced for a real logit: it is the image
// of one NaN bit pattern only).
__device__ __forceinline__ uint32_t cand_key_of(const float* scores, const int32_t* tokens, int L, int i) {
  const int t = tokens[i];
  const float x = scores[i];  // loaded with the token, not after it
  return (t >= 0 && t < L) ? ordered_key(x) : 0u;
}

__global__ void __launch_bounds__(kMThreads, 1)
    merge_kernel(const float* scores, const int32_t* tokens, int n, const int32_t* bt_row,
                 int max_pages, const int32_t* seq_len, int32_t* out) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  MergeSmem& s = *reinterpret_cast<MergeSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int L = row_len(seq_len, 0, max_pages, nullptr);
  if (L <= kTopK) {
    for (int i = tid; i < kTopK; i += kMThreads) out[i] = i < L ? physical_id(bt_row, i) : -1;
    return;
  }
  if (n <= kTopK) {
    // No more candidates than output slots (one rank's list): every real
    // one is selected; compacted in shared memory, then all slots written.
    if (tid == 0) s.out_count = 0;
    __syncthreads();
    for (int base = 0; base < n; base += kMThreads) {
      const int i = base + tid;
      const int t = i < n ? tokens[i] : -1;
      const bool real = t >= 0 && t < L;
      const int pos = warp_alloc_1(&s.out_count, real);
      if (real) s.cand_idx[pos] = physical_id(bt_row, t);
    }
    __syncthreads();
    const int cnt = s.out_count;
    for (int i = tid; i < kTopK; i += kMThreads) out[i] = i < cnt ? s.cand_idx[i] : -1;
    return;
  }
  // Slots stay -1 if the lists hold fewer than kTopK real entries.
  for (int i = tid; i < kTopK; i += kMThreads) out[i] = -1;
  for (int i = tid; i < kHistBins; i += kMThreads) s.hist[i] = 0u;
  if (tid == 0) {
    s.out_count = 0;
    s.cand_count = 0;
    s.eq_count = 0;
  }
  // The candidates' keys go to shared memory once, eight loads in flight per
  // thread, and every later pass reads them there (up to 8 ranks' lists).
  const bool staged = n <= kMergeStage;
  if (staged) {
    for (int base = 0; base < n; base += 8 * kMThreads) {
      uint32_t k[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = base + q * kMThreads + tid;
        k[q] = i < n ? cand_key_of(scores, tokens, L, i) : 0u;
      }
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = base + q * kMThreads + tid;
        if (i < n) s.key_all[i] = k[q];
      }
    }
  }
  auto key_of = [&](int i) -> uint32_t { return staged ? s.key_all[i] : cand_key_of(scores, tokens, L, i); };
  __syncthreads();
  for (int base = 0; base < n; base += kMThreads) {
    const int i = base + tid;
    const uint32_t key = i < n ? key_of(i) : 0u;
    hist_add(s.hist, key >> (32 - kHistBits), key != 0u);
  }
  __syncthreads();
  constexpr int kPer1 = kHistBins / kMThreads, kPer2 = kBins2 / kMThreads;
  uint32_t h1[kPer1];
#pragma unroll
  for (int i = 0; i < kPer1; ++i) h1[i] = s.hist[tid * kPer1 + i];
  find_threshold<kMThreads, kPer1>(s.sc, h1, kTopK);
  const uint32_t bin1 = static_cast<uint32_t>(s.sc.sel_bin);
  const int k1 = kTopK - s.sc.sel_above;
  const bool use_cand = s.sc.sel_count <= kCandCap;

  // Emit keys above the pivot bin; collect the pivot bin.
  for (int base = 0; base < n; base += kMThreads) {
    const int i = base + tid;
    const uint32_t key = i < n ? key_of(i) : 0u;
    const uint32_t bb = key >> (32 - kHistBits);
    const bool gt = key != 0u && bb > bin1;
    const bool eq = use_cand && key != 0u && bb == bin1;
    const int pos = warp_alloc_1(&s.out_count, gt);
    if (gt && pos < kTopK) out[pos] = physical_id(bt_row, tokens[i]);
    const int cpos = warp_alloc_1(&s.cand_count, eq);
    if (eq && cpos < kCandCap) {
      s.cand_key[cpos] = key;
      s.cand_idx[cpos] = i;
    }
  }
  __syncthreads();
  const int m = use_cand ? min(s.cand_count, kCandCap) : n;
  auto bucket = [&](int j) -> uint32_t {  // key of the j-th pivot-bin entry, or 0
    if (j >= m) return 0u;
    if (use_cand) return s.cand_key[j];
    const uint32_t key = key_of(j);
    return (key >> (32 - kHistBits)) == bin1 ? key : 0u;
  };
  auto index_of = [&](int j) { return use_cand ? s.cand_idx[j] : j; };

  for (int i = tid; i < kBins2; i += kMThreads) s.hist[i] = 0u;
  __syncthreads();
  for (int base = 0; base < m; base += kMThreads) {
    const uint32_t key = bucket(base + tid);
    if (key != 0u) atomicAdd(&s.hist[(key >> 10) & (kBins2 - 1)], 1u);
  }
  __syncthreads();
  uint32_t h2[kPer2];
#pragma unroll
  for (int i = 0; i < kPer2; ++i) h2[i] = s.hist[tid * kPer2 + i];
  find_threshold<kMThreads, kPer2>(s.sc, h2, k1);
  const uint32_t prefix2 = (bin1 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
  const int k2 = k1 - s.sc.sel_above;

  for (int i = tid; i < kBins2; i += kMThreads) s.hist[i] = 0u;
  __syncthreads();
  for (int base = 0; base < m; base += kMThreads) {
    const uint32_t key = bucket(base + tid);
    if (key != 0u && (key >> 10) == prefix2) atomicAdd(&s.hist[key & (kBins2 - 1)], 1u);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kPer2; ++i) h2[i] = s.hist[tid * kPer2 + i];
  find_threshold<kMThreads, kPer2>(s.sc, h2, k2);
  const uint32_t pivot = (prefix2 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
  const int k3 = k2 - s.sc.sel_above;

  for (int base = 0; base < m; base += kMThreads) {
    const int j = base + tid;
    const uint32_t key = bucket(j);
    const bool gt = key != 0u && key > pivot;
    const bool eq = key != 0u && key == pivot;
    const int pos = warp_alloc_1(&s.out_count, gt);
    if (gt && pos < kTopK) out[pos] = physical_id(bt_row, tokens[index_of(j)]);
    const int ticket = warp_alloc_1(&s.eq_count, eq);
    const int slot = kTopK - k3 + ticket;
    if (eq && ticket < k3 && slot >= 0 && slot < kTopK) out[slot] = physical_id(bt_row, tokens[index_of(j)]);
  }
}

// Rows that all fit in the top-K (max_pages * 64 <= 2048): the output is the
// physical ids of tokens 0..L-1 then -1, independent of q, K and weights
// (reference fast path, solution/python/kernel.cu:1050-1099).  One 128-thread
// CTA per row, 16-B stores.
__global__ void __launch_bounds__(128) short_rows_kernel(const int32_t* seq_lens,
                                                         const int32_t* block_table, int max_pages,
                                                         int32_t* out) {
  const int b = blockIdx.x;
  const int L = row_len(seq_lens, b, max_pages, nullptr);
  const int32_t* bt_row = block_table + static_cast<size_t>(b) * max_pages;
  int4* out4 = reinterpret_cast<int4*>(out + static_cast<size_t>(b) * kTopK);
  for (int v = threadIdx.x; v < kTopK / 4; v += 128) {
    const int t = 4 * v;
    int4 o;
    o.x = t + 0 < L ? physical_id(bt_row, t + 0) : -1;
    o.y = t + 1 < L ? physical_id(bt_row, t + 1) : -1;
    o.z = t + 2 < L ? physical_id(bt_row, t + 2) : -1;
    o.w = t + 3 < L ? physical_id(bt_row, t + 3) : -1;
    out4[v] = o;
  }
}

// Self-test of the bounded on-chip waits: waits on an mbarrier that nothing
// completes; the wait gives up after timeout_ns and reports
// DSAI_STATUS_WAIT_TIMEOUT, exactly as the indexer kernels do.
__global__ void wait_timeout_selftest_kernel(int* status, unsigned long long timeout_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    sm100::mbar_init(&bar, 1);
    sm100::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !sm100::mbar_wait(&bar, 0, nullptr, timeout_ns))
    report(status, DSAI_STATUS_WAIT_TIMEOUT);
}

bool g_attr_done[64];

cudaError_t ensure_attrs() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64 && g_attr_done[dev]) return cudaSuccess;
  e = cudaFuncSetAttribute(select_rows_kernel<true, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           row_smem_bytes<256>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(select_rows_kernel<false, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             row_smem_bytes<256>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(select_wide_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kWideSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(select_wide_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kWideSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMergeSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(select_split_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSplitSmemBytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(select_split_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSplitSmemBytes);
  // The split kernel's CTAs are small (21 KB): ask for the largest shared
  // memory carveout so that four of them fit on an SM (the driver may
  // otherwise size the carveout for fewer).
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(select_split_kernel<true>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(select_split_kernel<false>, cudaFuncAttributePreferredSharedMemoryCarveout,
                             cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) g_attr_done[dev] = true;
  return cudaSuccess;
}

}  // namespace

int select_smem_bytes() { return kWideSmemBytes; }

SelectShape select_shape(int rows, int max_pages, int sms) {
  SelectShape sh;
#if defined(DSAI_SELECT_FORCE_CLUSTER)
  const bool wide = false;
#elif defined(DSAI_SELECT_FORCE_WIDE)
  const bool wide = true;
#else
  // One wide CTA per row once the rows alone occupy a good share of the SMs.
  const bool wide = static_cast<long long>(rows) * 4 >= static_cast<long long>(sms) ||
                    static_cast<long long>(max_pages) * kPage <= kWideShortRow;
#endif
  if (wide) {
    sh.threads = kWThreads;
    sh.cluster = 1;
    return sh;
  }
  // As many CTAs per row as keep every CTA of the launch resident at once (at
  // most 8, a portable cluster), but no more than one per 1024 entries of the
  // longest possible row.
  const long long max_len = static_cast<long long>(max_pages) * kPage;
  const long long resident = static_cast<long long>(sms) * SelShape<256>::kCtasPerSm;
  long long c = rows > 0 ? resident / rows : 1;
  const long long useful = (max_len + 1023) / 1024;
  if (c > useful) c = useful;
  if (c > kMaxCluster) c = kMaxCluster;
  if (c < 1) c = 1;
  sh.threads = 256;
  sh.cluster = static_cast<int>(c);
  return sh;
}

// Whether the split kernel (several CTAs per row) may be used; with
// DSAI_SELECT=rows in the environment (read once) every call uses the
// one-CTA-per-row / one-cluster-per-row kernels instead (for comparison).
bool use_split_select() {
  static const bool split = [] {
    const char* v = getenv("DSAI_SELECT");
    return !(v && strcmp(v, "rows") == 0);
  }();
  return split;
}

cudaError_t launch_select_split(const SelectLaunch& p, long long chunks_per_row, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(static_cast<long long>(p.rows) * chunks_per_row));
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = kSplitSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int cpr = static_cast<int>(chunks_per_row);
  if (p.out_ids) return launch_kernel(cfg, select_split_kernel<true>, p, cpr);
  return launch_kernel(cfg, select_split_kernel<false>, p, cpr);
}

cudaError_t launch_select(const SelectLaunch& p, cudaStream_t stream) {
  cudaError_t e = ensure_attrs();
  if (e != cudaSuccess) return e;
  if (p.rows <= 0) return cudaSuccess;
  if (p.cand && use_split_select() && static_cast<long long>(p.rows) * 4 < static_cast<long long>(p.sms) &&
      static_cast<long long>(p.max_pages) * kPage > kWideShortRow) {
    // Few long rows: several CTAs per row.  (With many rows the
    // one-CTA-per-row kernel is faster: the split kernel's chain of dependent
    // steps per CTA — histogram, slot atomic, ticket, refinement — is longer
    // than the wide CTA's, measured 48.4 against 42.5 us per call at B = 64;
    // so it is for few short rows, whose logits one SM reads quickly: 14.2
    // against 16.4 us per call on config 0, 14.5 against 18.4 us at 14 rows of
    // up to 91 pages, CUDA-graph replays.)
    const long long max_len = static_cast<long long>(p.max_pages) * kPage;
    long long cpr = (max_len + kSChunk - 1) / kSChunk;
    if (cpr < 1) cpr = 1;
    if (static_cast<long long>(p.rows) * cpr <= 0x7FFFFFFFll) return launch_select_split(p, cpr, stream);
  }
  const SelectShape sh = select_shape(p.rows, p.max_pages, p.sms);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.rows) * static_cast<unsigned>(sh.cluster));
  cfg.blockDim = dim3(static_cast<unsigned>(sh.threads));
  cfg.dynamicSmemBytes = sh.threads == kWThreads ? kWideSmemBytes : row_smem_bytes<256>();
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = static_cast<unsigned>(sh.cluster);
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = sh.cluster > 1 ? 2 : 1;
  if (sh.threads == kWThreads) {
    if (p.out_ids) return launch_kernel(cfg, select_wide_kernel<true>, p);
    return launch_kernel(cfg, select_wide_kernel<false>, p);
  }
  if (p.out_ids) return launch_kernel(cfg, select_rows_kernel<true, 256>, p);
  return launch_kernel(cfg, select_rows_kernel<false, 256>, p);
}

cudaError_t launch_short_rows(const int32_t* seq_lens, const int32_t* block_table, int rows,
                              int max_pages, int32_t* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows));
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  return launch_kernel(cfg, short_rows_kernel, seq_lens, block_table, max_pages, out);
}

cudaError_t launch_wait_selftest(int* status, unsigned long long timeout_ns, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(status, timeout_ns);
  return cudaGetLastError();
}

cudaError_t launch_merge(const float* scores, const int32_t* tokens, int n_cand,
                         const int32_t* bt_row, int max_pages, const int32_t* seq_len,
                         int32_t* out, cudaStream_t stream) {
  cudaError_t e = ensure_attrs();
  if (e != cudaSuccess) return e;
  merge_kernel<<<1, kMThreads, kMergeSmemBytes, stream>>>(scores, tokens, n_cand, bt_row, max_pages,
                                                          seq_len, out);
  return cudaGetLastError();
}

}  // namespace dsai
