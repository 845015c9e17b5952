// select.cu — exact top-2048 selection over fp32 logits, and the merge of
// partial (score, token) candidate lists.
//
// Keys are the order-preserving u32 image of the fp32 logit, so "top-K by
// value" is "top-K by key".  Per row (one 512-thread CTA, two per SM):
//   digit 1  the histogram of the top 12 key bits (4096 bins) is the one the
//            scoring kernel accumulated for the row; the bin holding the
//            K-th largest key is found by a block suffix scan, and the
//            histogram is cleared for the next call;
//   pass     one vectorised pass over the row's logits: tokens in higher
//            bins are emitted directly, tokens in the pivot bin are
//            compacted into a shared-memory candidate list (<= 8192
//            entries; beyond that the refinement re-reads the row with a
//            prefix filter);
//   refine   10-bit + 10-bit histograms over the candidates give the exact
//            32-bit pivot; candidates above it are emitted, and ties at the
//            pivot fill the remaining slots in arbitrary order.
// Histogram updates are warp-aggregated with __match_any_sync (lanes holding
// the same bin add once), output slots are taken with one shared atomic per
// warp (in-warp scan).  The emitted set is exactly a top-K set of the
// logits; among equal logits at the boundary the choice is arbitrary, as in
// the reference's atomic emit (solution/python/kernel.cu:992-1018).
//
// Rows with seq_len <= 2048 emit ids of tokens 0..L-1 in token order and -1
// padding (reference kernel.cu:897-905, :1079-1097).
#include <cfloat>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace dsai {
namespace {

using sm100::grid_dep_launch_dependents;
using sm100::grid_dep_wait;

constexpr int kThreads = 512;
constexpr int kBins2 = 1024;   // 10-bit second and third digits
constexpr int kCandCap = 8192;
constexpr int kWarps = kThreads / 32;
constexpr int kUnroll = 8;     // float4 loads in flight per thread
constexpr int kBtCache = 4096; // block-table entries of a row kept in smem (rows <= 262144 tokens)

struct SelSmem {
  int32_t bt[kBtCache];
  uint32_t hist[kHistBins];
  uint32_t cand_key[kCandCap];
  int32_t cand_idx[kCandCap];
  int warp_tot[32];
  int warp_suf[32];
  uint32_t scan_total;
  int sel_bin;
  int sel_above;
  int out_count;
  int cand_count;
  int eq_count;
};

constexpr int kSmemBytes = static_cast<int>(sizeof(SelSmem));

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

// Finds the bin holding the k-th largest entry: sel_bin = bin with
// above(bin) < k <= above(bin) + hist[bin], sel_above = above(bin), where
// above(bin) counts entries in higher bins.  nbins is 4096 or 1024.  A
// two-level shuffle suffix scan (lanes, then the 32 warp totals).
__device__ void find_threshold(SelSmem& s, int nbins, int k) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = nbins / kThreads;
  const int lo = tid * per;
  constexpr int kMaxPer = kHistBins / kThreads;
  uint32_t h[kMaxPer];
  int sum = 0;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    h[i] = i < per ? s.hist[lo + i] : 0u;
    sum += static_cast<int>(h[i]);
  }
  int v = sum;  // inclusive suffix within the warp (higher lanes own higher bins)
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, v, off);
    if (lane + off < 32) v += y;
  }
  if (lane == 0) s.warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kWarps ? s.warp_tot[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_down_sync(0xffffffffu, t, off);
      if (lane + off < 32) t += y;
    }
    s.warp_suf[lane] = t;  // entries in warps >= lane
  }
  __syncthreads();
  int above = (warp < kWarps - 1 ? s.warp_suf[warp + 1] : 0) + (v - sum);
#pragma unroll
  for (int i = kMaxPer - 1; i >= 0; --i) {
    if (i < per) {
      const int hi = static_cast<int>(h[i]);
      if (above < k && above + hi >= k) {
        s.sel_bin = lo + i;
        s.sel_above = above;
      }
      above += hi;
    }
  }
  __syncthreads();
}

// Block-wide exclusive scan of a packed pair of counts (low / high 16 bits;
// the totals must stay below 65536).  Returns this thread's exclusive prefix
// and writes the block total to *total.
__device__ __forceinline__ uint32_t block_scan_packed(SelSmem& s, uint32_t v, uint32_t* total) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) s.warp_tot[warp] = static_cast<int>(incl);
  __syncthreads();
  if (warp == 0) {
    uint32_t t = lane < kWarps ? static_cast<uint32_t>(s.warp_tot[lane]) : 0u;
    uint32_t ti = t;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, ti, off);
      if (lane >= off) ti += y;
    }
    s.warp_suf[lane] = static_cast<int>(ti - t);  // exclusive prefix of warp totals
    if (lane == kWarps - 1) s.scan_total = ti;
  }
  __syncthreads();
  *total = s.scan_total;
  return static_cast<uint32_t>(s.warp_suf[warp]) + incl - v;
}

// Key sources.  key() == 0 means "no entry" (never produced for a real
// logit: it is the image of one NaN bit pattern only).
struct RowSrc {
  const float* row;
  __device__ __forceinline__ uint32_t key(int i) const { return ordered_key(row[i]); }
};
struct CandSrc {  // (score, token) list; padding (token -1) or tokens >= L are no entry
  const float* scores;
  const int32_t* tokens;
  int L;
  __device__ __forceinline__ uint32_t key(int i) const {
    const int t = tokens[i];
    return (t >= 0 && t < L) ? ordered_key(scores[i]) : 0u;
  }
};

// Output writers: i is the source index, key its key.
struct IdsOut {
  int32_t* out;
  const int32_t* bt_row;
  __device__ __forceinline__ void emit(int pos, int i, uint32_t) const {
    out[pos] = physical_id(bt_row, i);
  }
};
struct PairsOut {
  float* scores;
  int32_t* tokens;
  int32_t offset;
  __device__ __forceinline__ void emit(int pos, int i, uint32_t key) const {
    scores[pos] = key_to_float(key);
    tokens[pos] = i + offset;
  }
};
struct MergeOut {
  int32_t* out;
  const int32_t* bt_row;
  const int32_t* tokens;
  __device__ __forceinline__ void emit(int pos, int i, uint32_t) const {
    out[pos] = physical_id(bt_row, tokens[i]);
  }
};

// Emits keys above the pivot bin and compacts the pivot bin, for up to 4
// consecutive entries i0.. of this thread (cnt of them valid).
template <class Out>
__device__ __forceinline__ void classify(SelSmem& s, const Out& out, const uint32_t (&key)[4],
                                         int i0, int cnt, uint32_t bin1, bool use_cand) {
  int ngt = 0, neq = 0;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (u < cnt && key[u] != 0u) {
      const uint32_t b = key[u] >> (32 - kHistBits);
      ngt += b > bin1;
      neq += (use_cand && b == bin1);
    }
  }
  int pos = warp_alloc_n(&s.out_count, ngt);
  int cpos = warp_alloc_n(&s.cand_count, neq);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (u < cnt && key[u] != 0u) {
      const uint32_t b = key[u] >> (32 - kHistBits);
      if (b > bin1) {
        out.emit(pos++, i0 + u, key[u]);
      } else if (use_cand && b == bin1) {
        s.cand_key[cpos] = key[u];
        s.cand_idx[cpos] = i0 + u;
        ++cpos;
      }
    }
  }
}

// Selects the kTopK largest keys among src[0, n) (at least kTopK entries).
// g_hist: the 12-bit histogram of the entries accumulated by the producer of
// src (cleared here), or null to compute it.  VEC: the source is the 16-B
// aligned float row `row`, read with float4 loads.
template <bool VEC, class Src, class Out>
__device__ void select_topk(const Src& src, const float* row, const Out& out, int n,
                            uint32_t* g_hist, SelSmem& s) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    s.out_count = 0;
    s.cand_count = 0;
    s.eq_count = 0;
    s.sel_bin = 0;
    s.sel_above = 0;
  }
  if (g_hist) {
    static_assert(kHistBins == 8 * kThreads, "eight bins per thread");
    uint4* g4 = reinterpret_cast<uint4*>(g_hist);
    const uint4 h0 = g4[tid], h1 = g4[tid + kThreads];  // both loads in flight
    reinterpret_cast<uint4*>(s.hist)[tid] = h0;
    reinterpret_cast<uint4*>(s.hist)[tid + kThreads] = h1;
    g4[tid] = make_uint4(0u, 0u, 0u, 0u);  // clean for the next call
    g4[tid + kThreads] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
  } else {
    for (int i = tid; i < kHistBins; i += kThreads) s.hist[i] = 0u;
    __syncthreads();
    for (int base = 0; base < n; base += kThreads) {
      const int i = base + tid;
      const uint32_t key = i < n ? src.key(i) : 0u;
      hist_add(s.hist, key >> (32 - kHistBits), key != 0u);
    }
    __syncthreads();
  }
  find_threshold(s, kHistBins, kTopK);
  const uint32_t bin1 = static_cast<uint32_t>(s.sel_bin);
  const int k1 = kTopK - s.sel_above;
  const int n1 = static_cast<int>(s.hist[bin1]);
  const bool use_cand = n1 <= kCandCap;

  // One pass: emit above the pivot bin, compact the pivot bin.  Each chunk
  // gives every thread 32 consecutive-in-float4 entries; they are classified
  // into two bit masks (above the pivot bin / in it), the output slots come
  // from one block-wide scan of the mask popcounts, and only the set bits
  // (a few percent of the entries) are visited again, re-read through L1.
  if constexpr (VEC) {
    constexpr int kPer = 4 * kUnroll;  // entries per thread per chunk (32)
    static_assert(kPer == 32, "one mask bit per entry");
    const float4* row4 = reinterpret_cast<const float4*>(row);
    const int n4 = (n + 3) >> 2;       // the row buffer is padded to a multiple of 4
    int out_base = 0, cand_base = 0;
    for (int base4 = 0; base4 < n4; base4 += kThreads * kUnroll) {
      float4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int j = base4 + u * kThreads + tid;
        v[u] = j < n4 ? row4[j] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      uint32_t gtm = 0u, eqm = 0u;
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int i0 = 4 * (base4 + u * kThreads + tid);
        const float x[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const uint32_t b = ordered_key(x[c]) >> (32 - kHistBits);
          const bool in = i0 + c < n;
          gtm |= static_cast<uint32_t>(in && b > bin1) << (4 * u + c);
          eqm |= static_cast<uint32_t>(in && use_cand && b == bin1) << (4 * u + c);
        }
      }
      uint32_t tot;
      const uint32_t pre = block_scan_packed(s, __popc(gtm) | (__popc(eqm) << 16), &tot);
      int pos = out_base + static_cast<int>(pre & 0xFFFFu);
      int cpos = cand_base + static_cast<int>(pre >> 16);
      uint32_t m = gtm | eqm;
      while (m) {
        const int e = __ffs(m) - 1;
        m &= m - 1u;
        const int i = 4 * (base4 + (e >> 2) * kThreads + tid) + (e & 3);
        const uint32_t key = ordered_key(row[i]);  // L1 hit: loaded just above
        if ((gtm >> e) & 1u) {
          out.emit(pos++, i, key);
        } else {
          s.cand_key[cpos] = key;
          s.cand_idx[cpos] = i;
          ++cpos;
        }
      }
      out_base += static_cast<int>(tot & 0xFFFFu);
      cand_base += static_cast<int>(tot >> 16);
    }
    if (tid == 0) s.out_count = out_base;
  } else {
    for (int base = 0; base < n; base += kThreads) {
      const int i = base + tid;
      const uint32_t key[4] = {i < n ? src.key(i) : 0u, 0u, 0u, 0u};
      classify(s, out, key, i, i < n ? 1 : 0, bin1, use_cand);
    }
  }
  __syncthreads();

  // Entries of the pivot bin: the candidate list, or the source re-read.
  const int m = use_cand ? n1 : n;
  auto bucket = [&](int j, uint32_t& key, int& idx) {
    if (use_cand) {
      key = s.cand_key[j];
      idx = s.cand_idx[j];
    } else {
      key = src.key(j);
      idx = j;
      if (key == 0u || (key >> (32 - kHistBits)) != bin1) key = 0u;
    }
  };

  // refine: bits [10, 20)
  for (int i = tid; i < kBins2; i += kThreads) s.hist[i] = 0u;
  __syncthreads();
  for (int base = 0; base < m; base += kThreads) {
    const int j = base + tid;
    uint32_t key = 0u;
    int idx = 0;
    if (j < m) bucket(j, key, idx);
    hist_add(s.hist, (key >> 10) & 1023u, key != 0u);
  }
  __syncthreads();
  find_threshold(s, kBins2, k1);
  const uint32_t bin2 = static_cast<uint32_t>(s.sel_bin);
  const int k2 = k1 - s.sel_above;
  const uint32_t prefix2 = (bin1 << 10) | bin2;

  // refine: bits [0, 10)
  for (int i = tid; i < kBins2; i += kThreads) s.hist[i] = 0u;
  __syncthreads();
  for (int base = 0; base < m; base += kThreads) {
    const int j = base + tid;
    uint32_t key = 0u;
    int idx = 0;
    if (j < m) bucket(j, key, idx);
    hist_add(s.hist, key & 1023u, key != 0u && (key >> 10) == prefix2);
  }
  __syncthreads();
  find_threshold(s, kBins2, k2);
  const uint32_t pivot = (prefix2 << 10) | static_cast<uint32_t>(s.sel_bin);
  const int k3 = k2 - s.sel_above;  // how many keys equal to the pivot are taken

  for (int base = 0; base < m; base += kThreads) {
    const int j = base + tid;
    uint32_t key = 0u;
    int idx = 0;
    if (j < m) bucket(j, key, idx);
    const bool gt = key != 0u && key > pivot;
    const bool eq = key != 0u && key == pivot;
    const int pos = warp_alloc_n(&s.out_count, gt ? 1 : 0);
    if (gt) out.emit(pos, idx, key);
    const int ticket = warp_alloc_n(&s.eq_count, eq ? 1 : 0);
    if (eq && ticket < k3) out.emit(kTopK - k3 + ticket, idx, key);
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1) select_kernel(SelectLaunch p) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelSmem& s = *reinterpret_cast<SelSmem*>(smem_raw);
  // Launched as a programmatic dependent of the scoring kernel: wait for its
  // logits and histograms, then let the next grid start launching.
  grid_dep_wait();
  grid_dep_launch_dependents();
  const int b = blockIdx.x;
  const int L = row_len(p.seq_lens, b, p.max_pages, nullptr);
  const int32_t* bt_row = p.block_table + static_cast<size_t>(b) * p.max_pages;
  const float* row = p.logits + static_cast<size_t>(b) * p.ld;
  uint32_t* g_hist = p.hist + static_cast<size_t>(b) * kHistBins;

  if (p.out_ids) {
    int32_t* out = p.out_ids + static_cast<size_t>(b) * kTopK;
    if (L <= kTopK) {
      for (int i = threadIdx.x; i < kTopK; i += kThreads) out[i] = i < L ? physical_id(bt_row, i) : -1;
      return;
    }
    // The row's block table in shared memory: emitting an id then costs no
    // dependent global load.
    const int npages = (L + kPage - 1) / kPage;
    const int32_t* bt_ids = bt_row;
    if (npages <= kBtCache) {
      for (int i = threadIdx.x; i < npages; i += kThreads) s.bt[i] = bt_row[i];
      bt_ids = s.bt;  // made visible by the barrier inside select_topk
    }
    select_topk<true>(RowSrc{row}, row, IdsOut{out, bt_ids}, L, g_hist, s);
  } else {
    float* sc = p.out_scores + static_cast<size_t>(b) * kTopK;
    int32_t* tk = p.out_tokens + static_cast<size_t>(b) * kTopK;
    if (L <= kTopK) {
      for (int i = threadIdx.x; i < kTopK; i += kThreads) {
        sc[i] = i < L ? row[i] : -INFINITY;
        tk[i] = i < L ? i + p.token_offset : -1;
      }
      return;
    }
    select_topk<true>(RowSrc{row}, row, PairsOut{sc, tk, p.token_offset}, L, g_hist, s);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
    merge_kernel(const float* scores, const int32_t* tokens, int n_cand, const int32_t* bt_row,
                 int max_pages, const int32_t* seq_len, int32_t* out) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SelSmem& s = *reinterpret_cast<SelSmem*>(smem_raw);
  const int L = row_len(seq_len, 0, max_pages, nullptr);
  if (L <= kTopK) {
    for (int i = threadIdx.x; i < kTopK; i += kThreads) out[i] = i < L ? physical_id(bt_row, i) : -1;
    return;
  }
  // Slots stay -1 if the candidates hold fewer than kTopK real entries.
  for (int i = threadIdx.x; i < kTopK; i += kThreads) out[i] = -1;
  __syncthreads();
  select_topk<false>(CandSrc{scores, tokens, L}, nullptr, MergeOut{out, bt_row, tokens}, n_cand,
                     nullptr, s);
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
  e = cudaFuncSetAttribute(select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  if (e != cudaSuccess) return e;
  if (dev >= 0 && dev < 64) g_attr_done[dev] = true;
  return cudaSuccess;
}

}  // namespace

int select_smem_bytes() { return kSmemBytes; }

cudaError_t launch_select(const SelectLaunch& p, cudaStream_t stream) {
  cudaError_t e = ensure_attrs();
  if (e != cudaSuccess) return e;
  if (p.rows <= 0) return cudaSuccess;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.rows);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, select_kernel, p);
}

cudaError_t launch_short_rows(const int32_t* seq_lens, const int32_t* block_table, int rows,
                              int max_pages, int32_t* out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  short_rows_kernel<<<rows, 128, 0, stream>>>(seq_lens, block_table, max_pages, out);
  return cudaGetLastError();
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
  merge_kernel<<<1, kThreads, kSmemBytes, stream>>>(scores, tokens, n_cand, bt_row, max_pages,
                                                    seq_len, out);
  return cudaGetLastError();
}

}  // namespace dsai
