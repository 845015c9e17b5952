// fused.cu — scoring and top-2048 selection of a batch of many rows in one
// persistent launch.
//
// The two-launch path (score_kernel, then select_wide_kernel) leaves HBM idle
// while the selection runs: every scorer CTA's slice spans the whole call, so
// every row is complete only when the last scorer CTA ends, and only then can
// the selection of any row start.  Here one grid of one CTA per SM does both:
//
//   scorer CTAs   two independent copies of score_kernel's pipeline per CTA
//                 (per copy: TMA producer warp, one tcgen05 MMA issuer, four
//                 epilogue warps, a 5-stage K ring and 256 TMEM columns;
//                 identical arithmetic, so the logits are bit-identical), over
//                 an interleaved schedule: the flat tile sequence is cut into
//                 chunks of `chunk` tiles and pipeline s of S takes chunks
//                 s, s + S, s + 2S, ...  All pipelines move through the
//                 sequence together, so rows complete one after another during
//                 the call.  Rows are laid out longest first (up to 256 rows):
//                 the rows that complete last are the cheapest to select.  An
//                 epilogue warp adds the tiles it finished to its row's
//                 counter with a fire-and-forget reduction when it leaves the
//                 row (no fence on the scoring path).
//   selector CTAs a whole SM each (384 threads, the shared memory of both
//                 pipelines): they take rows in the scoring order (one atomic
//                 per row), wait for the row's counter to reach its total,
//                 and run the exact radix top-2048 of select_wide_kernel over
//                 the row's histogram and logits, which the L2 holds.
//                 Because the scorers publish without fences, a selector
//                 checks the data itself: the histogram must sum to the row's
//                 length (every reduction landed) and no logit may still hold
//                 the sentinel bit pattern the logits buffer is filled with
//                 between calls (every store landed); it re-reads otherwise.
//                 It writes the sentinel back over the row's logits, and
//                 clears the row's histogram and counter for the next call.
//                 Selectors also write the rows that fit in the top-K.
//
// Scorers never wait for selectors; selectors wait (bounded) only for rows
// that scorers, all resident or scheduled as soon as any CTA retires, will
// finish.  The row-claim and exit counters live in the workspace header and
// are reset by the last selector to leave.  A call that gave up a wait
// (DSAI_STATUS_WAIT_TIMEOUT) may leave counters, histograms or the sentinel
// incomplete: initialize the workspace again (dsai_workspace_init) before
// its next use.
//
// Opt-in (DSAI_FUSED=1 in the environment).
#include <cstdlib>

#include "common.cuh"
#include "launch.h"
#include "radix.cuh"
#include "sm100.cuh"
#include "tiles.cuh"

namespace dsai {
namespace {

using namespace sm100;
using namespace radix;

constexpr int kFThreads = 384;               // two scoring pipelines of 6 warps
constexpr int kFPipes = 2;
constexpr int kFPipeWarps = 6;
constexpr int kFStages = 5;
constexpr int kFScaleSlots = 12;             // > 9: producer runs <= 5 K stages + 4 accumulators ahead
constexpr int kFAccs = 4;
constexpr int kFAccCols = kHeads;
constexpr int kFPipeTmemCols = kFAccs * kFAccCols;       // 256 per pipeline
constexpr int kFTmemCols = kFPipes * kFPipeTmemCols;     // 512
constexpr int kFEpiWarps = 4;
constexpr uint32_t kFScaleTx = kPage * 4;
constexpr int kFSortRows = 256;              // rows laid out longest first up to this many
constexpr int kFMaxPer = (kMaxRowsPerLaunch + kFThreads - 1) / kFThreads;

// Selector shape: 32 entries per thread and round, two rounds in flight.
constexpr int kFPer = 32;
constexpr int kFRound = kFThreads * kFPer;   // 12288 entries (48 KB) per round
constexpr int kFRing = 2;
constexpr int kFCap = 8192;                  // pivot-bin keys kept in shared memory
constexpr int kFBtCache = 2048;              // block-table entries of a row in smem (131072 tokens)
constexpr int kFSmall = 64;
constexpr int kFH1Threads = 256;             // 16 first-digit bins each
constexpr int kFH2Threads = 256;             // 4 second-digit bins each

// Logits buffer contents between calls: this bit pattern (a NaN arithmetic
// never produces on this GPU; the scorer maps it to another NaN) marks
// entries not yet written by the current call.
constexpr uint32_t kSentinel = 0xFFFFFFFFu;

// Control words in the workspace header (int offsets, 64 B apart; the status
// word is int 0): next row position to take, selectors done.
constexpr int kCtlHead = 16;
constexpr int kCtlFin = 48;
// Per-row word after the row's 4096 histogram bins: warp-tiles finished
// (4 epilogue warps x the row's tiles when complete).
constexpr int kRowDone = kHistBins + 2;

struct FusedParams {
  const float* weights;
  const int32_t* seq_lens;
  const int32_t* block_table;
  float* logits;      // sentinel-filled on entry; left so (unless keep_logits)
  uint32_t* hist;     // [rows, kHistStride]: bins and counters zero on entry, left zero
  int* ws;            // workspace header: status word, control words
  int32_t* out_ids;
  int rows;
  int max_pages;
  int num_pages;
  int ld;
  int score_all;
  int keep_logits;    // 1: leave the logits (a caller's buffer), 0: restore the sentinel
  int scorers;        // CTAs [0, scorers) score, the others select
  int chunk;          // tiles per chunk of the interleaved schedule
};

struct alignas(1024) PipeSmem {
  uint8_t k[kFStages][2 * kPageKBytes];  // 1024-B aligned stages, SW128 K-major
  uint8_t q[2][kQBytes];
  float w[2][kHeads];                    // the row's head weights, with its query
  float scale[kFScaleSlots][kTileTok];
  uint64_t full[kFStages];
  uint64_t empty[kFStages];
  uint64_t sfull[kFScaleSlots];
  uint64_t sempty[kFScaleSlots];
  uint64_t qfull[2];
  uint64_t qempty[2];
  uint64_t tfull[kFAccs];
  uint64_t tempty[kFAccs];
  uint64_t drain;
  int abort;
};

struct SelectorSmem {
  float4 vals[kFRing][kFPer / 4][kFThreads];  // two rounds of logits
  uint32_t cand_key[kFCap];                   // keys in the pivot bin and their ids
  int32_t cand_val[kFCap];
  uint32_t hist[kBins2];                      // second (then third) digit histogram
  int32_t bt[kFBtCache];                      // the row's pages
  uint32_t small_key[kFSmall];
  int32_t small_val[kFSmall];
  Scan sc;
  int out_count;
  int cand_count;
  int small_count;
  int eq_count;
  int extreme[2];                             // first-digit bins 0 and 4088..4095 are not empty
  int item;                                   // the row taken (-1: none left)
  int hist_done;
};

struct FusedSmem {
  union {
    PipeSmem pipe[kFPipes];
    SelectorSmem se;
  } u;
  uint32_t tmem_base;
  int warp_sums[kFThreads / 32];
  uint16_t order[kMaxRowsPerLaunch];      // row of each position of the tile sequence
  int row_start[kMaxRowsPerLaunch + 1];   // first tile of each position
};

constexpr int kFSmemBytes = static_cast<int>(sizeof(FusedSmem)) + 1024;
static_assert(kFSmemBytes <= 232448, "one fused CTA per SM must fit");
static_assert(sizeof(PipeSmem) % 1024 == 0, "both pipelines' K rings 1024-B aligned");
static_assert(kFH1Threads * 16 == kHistBins && kFH2Threads * 4 == kBins2, "bin ownership");
static_assert(kFSmall <= kFThreads && kFH1Threads <= kFThreads, "selector shape");
static_assert(kFPer / 4 == 8, "eight float4 per thread and round");

__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fail(PipeSmem& s, int* status) {
  report(status, DSAI_STATUS_WAIT_TIMEOUT);
  *reinterpret_cast<volatile int*>(&s.abort) = 1;
}

// Row order (longest first when rows <= kFSortRows, ties by row index; else
// the natural order) and the exclusive prefix of the tiles of the rows in
// that order (all threads).
__device__ void build_order(FusedSmem& s, const FusedParams& p) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int* lens = s.row_start;  // scratch, rebuilt below
  int* st = blockIdx.x == 0 ? p.ws : nullptr;
  for (int b = tid; b < p.rows; b += kFThreads) lens[b] = row_len(p.seq_lens, b, p.max_pages, st);
  __syncthreads();
  if (p.rows <= kFSortRows) {
    for (int b = tid; b < p.rows; b += kFThreads) {
      const int Lb = lens[b];
      int r = 0;
      for (int c = 0; c < p.rows; ++c) {
        const int Lc = lens[c];
        r += (Lc > Lb || (Lc == Lb && c < b)) ? 1 : 0;
      }
      s.order[r] = static_cast<uint16_t>(b);
    }
  } else {
    for (int b = tid; b < p.rows; b += kFThreads) s.order[b] = static_cast<uint16_t>(b);
  }
  __syncthreads();
  const int per = (p.rows + kFThreads - 1) / kFThreads;
  const int i0 = min(p.rows, tid * per), i1 = min(p.rows, i0 + per);
  int tl[kFMaxPer];
  int sum = 0;
#pragma unroll
  for (int k = 0; k < kFMaxPer; ++k) {
    const int i = i0 + k;
    tl[k] = i < i1 ? row_tiles(lens[s.order[i]], p.score_all != 0) : 0;
    sum += tl[k];
  }
  int incl = sum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) s.warp_sums[warp] = incl;
  __syncthreads();  // also: every thread has read `lens` before it is overwritten
  int prefix = incl - sum;
  for (int w = 0; w < warp; ++w) prefix += s.warp_sums[w];
#pragma unroll
  for (int k = 0; k < kFMaxPer; ++k) {
    const int i = i0 + k;
    if (i < i1) s.row_start[i] = prefix;
    prefix += tl[k];
  }
  if (tid == kFThreads - 1) s.row_start[p.rows] = prefix;
  __syncthreads();
}

// The tiles of pipeline s of S: chunks s, s + S, ... of `chunk` tiles each
// over the T tiles of the sequence; local tile j is global tile tile(j).
struct Sched {
  int s, S, C, n;
  __device__ void init(int s_, int S_, int C_, int T) {
    s = s_;
    S = S_;
    C = C_;
    const int NC = (T + C - 1) / C;
    const int my = s < NC ? (NC - 1 - s) / S + 1 : 0;
    n = my * C;
    if (my > 0 && s + (my - 1) * S == NC - 1) n -= NC * C - T;  // the partial last chunk
  }
  __device__ __forceinline__ int tile(int j) const { return ((j / C) * S + s) * C + (j % C); }
};

// Walks a pipeline's tiles: the position of the tile's row in the sequence,
// the tile's index inside the row, the row's end.
struct FCursor {
  int j, t, pos, jr, end;
  __device__ void seek(const int* rs, int rows, int tt) {
    t = tt;
    pos = find_row(rs, rows, tt);
    jr = tt - rs[pos];
    end = rs[pos + 1];
  }
  __device__ void start(const int* rs, int rows, const Sched& sc) {
    j = 0;
    if (sc.n > 0) seek(rs, rows, sc.tile(0));
  }
  __device__ void advance(const int* rs, int rows, const Sched& sc) {
    ++j;
    if (j >= sc.n) return;
    const int tt = sc.tile(j);
    if (tt == t + 1 && tt < end) {
      t = tt;
      ++jr;
    } else {
      seek(rs, rows, tt);
    }
  }
};

struct TileRef {
  int pos, pg0, pg1, two;
};

__device__ __forceinline__ TileRef resolve_tile(const FusedSmem& s, const FusedParams& p, int t) {
  TileRef r;
  r.pos = find_row(s.row_start, p.rows, t);
  const int b = s.order[r.pos];
  const int j = t - s.row_start[r.pos];
  const int32_t* bt = p.block_table + static_cast<size_t>(b) * p.max_pages;
  const int L = row_len(p.seq_lens, b, p.max_pages, nullptr);
  r.pg0 = bt[2 * j];
  r.pg1 = (2 * j + 1 < p.max_pages) ? bt[2 * j + 1] : 0;
  r.two = (2 * j + 1) * kPage < L;
  return r;
}

// ---------------------------------------------------------------- scorer

// One scoring pipeline: warps [6*pipe, 6*pipe + 6) of the CTA, its own
// shared memory and TMEM columns, scoring pipeline index `gp` of `npipes`.
__device__ void pipe_role(FusedSmem& sm, PipeSmem& s, uint32_t tmem, const CUtensorMap* tmap_q,
                          const CUtensorMap* tmap_k, const CUtensorMap* tmap_s, const FusedParams& p,
                          int gp, int npipes) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int role = warp % kFPipeWarps;
  const int* rs = sm.row_start;
  Sched sched;
  sched.init(gp, npipes, p.chunk, rs[p.rows]);
  if (sched.n <= 0) return;

  if (role == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_k = l2_policy_evict_first();
    const uint64_t pol_q = l2_policy_evict_last();
    int stage = 0, sslot = 0, qs = 1, cur_pos = -1;
    uint32_t phase = 0, sphase = 0;
    uint32_t qe_par[2] = {0u, 0u};
    int q_uses[2] = {0, 0};
    int k_fills = 0, s_fills = 0;
    bool ok = true;
    TileRef nxt = {0, 0, 0, 0};
    if (lane < sched.n) nxt = resolve_tile(sm, p, sched.tile(lane));
    for (int jb = 0; jb < sched.n && ok; jb += 32) {
      const TileRef cur = nxt;
      if (jb + 32 + lane < sched.n) nxt = resolve_tile(sm, p, sched.tile(jb + 32 + lane));
      if (jb + lane < sched.n &&
          (static_cast<unsigned>(cur.pg0) >= static_cast<unsigned>(p.num_pages) ||
           (cur.two && static_cast<unsigned>(cur.pg1) >= static_cast<unsigned>(p.num_pages))))
        report(p.ws, DSAI_STATUS_BAD_PAGE);  // TMA zero-fills out-of-range pages
      const int n = min(32, sched.n - jb);
      for (int i = 0; i < n; ++i) {
        const int ps = __shfl_sync(0xffffffffu, cur.pos, i);
        const int a = __shfl_sync(0xffffffffu, cur.pg0, i);
        const int b = __shfl_sync(0xffffffffu, cur.pg1, i);
        const int tw = __shfl_sync(0xffffffffu, cur.two, i);
        int good = 1;
        if (lane == 0) {
          if (ps != cur_pos) {
            cur_pos = ps;
            qs ^= 1;
            // The slot is free once the MMAs of its last row completed and
            // every epilogue warp took that row's weights.
            if (!mbar_wait(&s.qempty[qs], qe_par[qs] ^ 1u, &s.abort, kWaitTimeoutNs)) {
              good = 0;
            } else {
              qe_par[qs] ^= 1u;
              ++q_uses[qs];
              const int row = sm.order[ps];
              mbar_arrive_expect_tx(&s.qfull[qs], kQBytes + kHeads * 4);
              tma_load_2d(s.q[qs], tmap_q, &s.qfull[qs], 0, row * kHeads, pol_q);
              bulk_load(s.w[qs], p.weights + static_cast<size_t>(row) * kHeads, kHeads * 4, &s.qfull[qs], pol_q);
            }
          }
          if (good && !mbar_wait(&s.empty[stage], phase ^ 1u, &s.abort, kWaitTimeoutNs)) good = 0;
          if (good && !mbar_wait(&s.sempty[sslot], sphase ^ 1u, &s.abort, kWaitTimeoutNs)) good = 0;
          if (good) {
            mbar_arrive_expect_tx(&s.full[stage], tw ? 2 * kPageKBytes : kPageKBytes);
            mbar_arrive_expect_tx(&s.sfull[sslot], tw ? 2 * kFScaleTx : kFScaleTx);
            tma_load_3d(s.k[stage], tmap_k, &s.full[stage], 0, 0, a, pol_k);
            tma_load_2d(s.scale[sslot], tmap_s, &s.sfull[sslot], 0, a, pol_k);
            if (tw) {
              tma_load_3d(s.k[stage] + kPageKBytes, tmap_k, &s.full[stage], 0, 0, b, pol_k);
              tma_load_2d(s.scale[sslot] + kPage, tmap_s, &s.sfull[sslot], 0, b, pol_k);
            }
            ++k_fills;
            ++s_fills;
            if (++stage == kFStages) { stage = 0; phase ^= 1u; }
            if (++sslot == kFScaleSlots) { sslot = 0; sphase ^= 1u; }
          } else {
            fail(s, p.ws);
          }
        }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) { ok = false; break; }
      }
    }
    // Never leave with a TMA in flight: wait for the latest fill of every slot.
    if (lane == 0) {
      for (int i = 0; i < kFStages && i < k_fills; ++i) {
        const int last = k_fills - 1 - i;
        if (!mbar_wait(&s.full[last % kFStages], (last / kFStages) & 1, nullptr, kWaitTimeoutNs))
          report(p.ws, DSAI_STATUS_WAIT_TIMEOUT);
      }
      for (int i = 0; i < kFScaleSlots && i < s_fills; ++i) {
        const int last = s_fills - 1 - i;
        if (!mbar_wait(&s.sfull[last % kFScaleSlots], (last / kFScaleSlots) & 1, nullptr, kWaitTimeoutNs))
          report(p.ws, DSAI_STATUS_WAIT_TIMEOUT);
      }
      for (int i = 0; i < 2; ++i)
        if (q_uses[i] > 0 && !mbar_wait(&s.qfull[i], (q_uses[i] - 1) & 1, nullptr, kWaitTimeoutNs))
          report(p.ws, DSAI_STATUS_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else if (role == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_e4m3_f32(kTileTok, kHeads);
      int stage = 0, acc = 0, qs = 1, cur_pos = -1;
      uint32_t phase = 0, aphase = 0;
      uint32_t qf_par[2] = {0u, 0u};
      FCursor c;
      c.start(rs, p.rows, sched);
      for (; c.j < sched.n; c.advance(rs, p.rows, sched)) {
        if (c.pos != cur_pos) {
          if (cur_pos >= 0) umma_commit(&s.qempty[qs]);  // previous row's Q free when done
          cur_pos = c.pos;
          qs ^= 1;
          if (!mbar_wait(&s.qfull[qs], qf_par[qs], &s.abort, kWaitTimeoutNs)) { fail(s, p.ws); break; }
          qf_par[qs] ^= 1u;
        }
        if (!mbar_wait(&s.full[stage], phase, &s.abort, kWaitTimeoutNs)) { fail(s, p.ws); break; }
        if (!mbar_wait(&s.tempty[acc], aphase ^ 1u, &s.abort, kWaitTimeoutNs)) { fail(s, p.ws); break; }
        tc_fence_after();
        const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(s.k[stage]));
        const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(s.q[qs]));
        const uint32_t d = tmem + static_cast<uint32_t>(acc * kFAccCols);
#pragma unroll
        for (int kk = 0; kk < kDim / 32; ++kk)  // K = 32 e4m3 (32 B) per MMA
          umma_f8(d, adesc + 2u * kk, bdesc + 2u * kk, idesc, kk > 0 ? 1u : 0u);
        umma_commit(&s.empty[stage]);
        umma_commit(&s.tfull[acc]);
        if (++stage == kFStages) { stage = 0; phase ^= 1u; }
        if (++acc == kFAccs) { acc = 0; aphase ^= 1u; }
      }
      umma_commit(&s.drain);
      if (!mbar_wait(&s.drain, 0, nullptr, kWaitTimeoutNs)) report(p.ws, DSAI_STATUS_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;              // TMEM lanes [32*quad, 32*quad+32)
    const int tok = quad * 32 + lane;       // token of the tile owned by this thread
    int acc = 0, sslot = 0, qs = 1, cur_pos = -1, cur_row = 0, L = 0, pending = 0;
    uint32_t aphase = 0, sphase = 0;
    uint32_t qf_par[2] = {0u, 0u};
    bool hist_row = false;
    float w[kHeads];
    float* out_row = nullptr;
    uint32_t* hist_g = nullptr;
    // Publishes this warp's finished tiles of the current row (no fence: a
    // selector checks that the row's data landed before it uses it).
    auto flush = [&]() {
      if (hist_row && pending > 0) {
        __syncwarp();
        if (lane == 0) atomicAdd(hist_g + kRowDone, static_cast<uint32_t>(pending));  // RED
      }
      pending = 0;
    };
    FCursor c;
    c.start(rs, p.rows, sched);
    bool ok = true;
    for (; c.j < sched.n; c.advance(rs, p.rows, sched)) {
      if (c.pos != cur_pos) {
        flush();
        cur_pos = c.pos;
        cur_row = sm.order[cur_pos];
        qs ^= 1;
        // The row's weights came with its query (the MMA issuer saw the slot
        // fill; this wait makes the copy visible to this warp too).
        if (!__all_sync(0xffffffffu, mbar_wait(&s.qfull[qs], qf_par[qs], &s.abort, kWaitTimeoutNs))) {
          fail(s, p.ws);
          ok = false;
          break;
        }
        qf_par[qs] ^= 1u;
        const float4* w4 = reinterpret_cast<const float4*>(s.w[qs]);
#pragma unroll
        for (int i = 0; i < kHeads / 4; ++i) {
          const float4 v = w4[i];
          w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.qempty[qs]);
        L = row_len(p.seq_lens, cur_row, p.max_pages, nullptr);
        hist_row = L > kTopK;  // only rows that go through the radix select
        out_row = p.logits + static_cast<size_t>(cur_row) * p.ld;
        hist_g = p.hist + static_cast<size_t>(cur_row) * kHistStride;
      }
      if (!__all_sync(0xffffffffu, mbar_wait(&s.tfull[acc], aphase, &s.abort, kWaitTimeoutNs))) {
        fail(s, p.ws);
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r0[32], r1[32];
      const uint32_t taddr = tmem + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * kFAccCols);
      tmem_ld_32x32b_x32(taddr, r0);
      tmem_ld_32x32b_x32(taddr + 32u, r1);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.tempty[acc]);
      if (!__all_sync(0xffffffffu, mbar_wait(&s.sfull[sslot], sphase, &s.abort, kWaitTimeoutNs))) {
        fail(s, p.ws);
        ok = false;
        break;
      }
      const float sc = s.scale[sslot][tok];
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.sempty[sslot]);
      // The per-row scorer's summation order (bit-identical logits).
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f, b0 = 0.f, b1 = 0.f, b2 = 0.f, b3 = 0.f;
#pragma unroll
      for (int h = 0; h < 32; h += 4) {
        a0 = fmaf(fmaxf(__uint_as_float(r0[h + 0]), 0.f), w[h + 0], a0);
        a1 = fmaf(fmaxf(__uint_as_float(r0[h + 1]), 0.f), w[h + 1], a1);
        a2 = fmaf(fmaxf(__uint_as_float(r0[h + 2]), 0.f), w[h + 2], a2);
        a3 = fmaf(fmaxf(__uint_as_float(r0[h + 3]), 0.f), w[h + 3], a3);
        b0 = fmaf(fmaxf(__uint_as_float(r1[h + 0]), 0.f), w[32 + h + 0], b0);
        b1 = fmaf(fmaxf(__uint_as_float(r1[h + 1]), 0.f), w[32 + h + 1], b1);
        b2 = fmaf(fmaxf(__uint_as_float(r1[h + 2]), 0.f), w[32 + h + 2], b2);
        b3 = fmaf(fmaxf(__uint_as_float(r1[h + 3]), 0.f), w[32 + h + 3], b3);
      }
      float logit = (((a0 + b0) + (a1 + b1)) + ((a2 + b2) + (a3 + b3))) * sc;
      if (__float_as_uint(logit) == kSentinel) logit = __uint_as_float(0x7FFFFFFFu);
      const int t_abs = c.jr * kTileTok + tok;
      const bool live = t_abs < L;
      if (live) out_row[t_abs] = logit;
      if (hist_row) {
        const uint32_t bin = ordered_key(logit) >> (32 - kHistBits);
        const unsigned act = __ballot_sync(0xffffffffu, live);
        if (live) {
          const unsigned peers = __match_any_sync(act, bin);
          if (lane == __ffs(peers) - 1) atomicAdd(hist_g + bin, static_cast<uint32_t>(__popc(peers)));  // RED
        }
      }
      ++pending;
      if (++acc == kFAccs) { acc = 0; aphase ^= 1u; }
      if (++sslot == kFScaleSlots) { sslot = 0; sphase ^= 1u; }
    }
    if (ok) flush();  // an aborted warp leaves its row incomplete (its selector times out)
  }
}

// ---------------------------------------------------------------- selector

// A float4 of the row's logits whose valid entries (mask bits) still hold
// the sentinel is re-read from L2 until every valid entry has landed
// (bounded; false on timeout).
__device__ __forceinline__ bool settle(float4& w, const float* src, uint32_t valid) {
  auto waiting = [&](const float4& v) {
    return ((valid & 1u) && __float_as_uint(v.x) == kSentinel) || ((valid & 2u) && __float_as_uint(v.y) == kSentinel) ||
           ((valid & 4u) && __float_as_uint(v.z) == kSentinel) || ((valid & 8u) && __float_as_uint(v.w) == kSentinel);
  };
  if (!waiting(w)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
    __nanosleep(64);
    w = __ldcg(reinterpret_cast<const float4*>(src));
    if (!waiting(w)) return true;
    if (global_timer_ns() - t0 > kWaitTimeoutNs) return false;
  }
}

// The exact top-2048 of one completed row (kIds form of select_wide_kernel,
// 384 threads): digit 1 from the row's histogram, one pass over the logits
// (keys above the pivot bin to the output, keys in it to a list and the
// second-digit histogram), then digits 2 and 3 over the list.  Clears the
// row's histogram and counter; restores the sentinel over its logits.
__device__ void select_row(SelectorSmem& s, const FusedParams& p, int b) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L = row_len(p.seq_lens, b, p.max_pages, nullptr);
  const int32_t* bt_row = p.block_table + static_cast<size_t>(b) * p.max_pages;
  float* row = p.logits + static_cast<size_t>(b) * p.ld;
  RowOut<true> out;
  out.ids = p.out_ids + static_cast<size_t>(b) * kTopK;
  out.scores = nullptr;
  out.tokens = nullptr;
  out.offset = 0;
  uint32_t* g_hist = p.hist + static_cast<size_t>(b) * kHistStride;
  if (tid == 0) {
    s.out_count = 0;
    s.cand_count = 0;
    s.small_count = 0;
    s.eq_count = 0;
  }
  const int npg = (L + kPage - 1) / kPage;
  const bool bt_cached = npg <= kFBtCache;
  if (bt_cached)
    for (int i = tid; i < npg; i += kFThreads) s.bt[i] = bt_row[i];
  for (int i = tid; i < kBins2; i += kFThreads) s.hist[i] = 0u;

  // Round r of logits (entries [r*kFRound, (r+1)*kFRound)) into ring slot
  // r % kFRing (L2 only), one cp.async group per round; each thread reads
  // only its own entries.  Entries past the row's end are zero-filled.
  const int nrounds = (L + kFRound - 1) / kFRound;
  auto load_round = [&](int r) {
    const int base = r * kFRound;
    const int n = L - base;
    float4(*v)[kFThreads] = s.vals[r % kFRing];
#pragma unroll
    for (int u = 0; u < kFPer / 4; ++u) {
      const int e = u * 4 * kFThreads + 4 * tid;
      cp_async_16(&v[u][tid], e < n ? row + base + e : row, e < n ? 16u : 0u);
    }
    cp_async_commit_group();
  };
#pragma unroll
  for (int r = 0; r < kFRing; ++r) load_round(r);

  // Digit 1: threads < 256 own 16 bins each, read from L2.  The bins must
  // add up to the row's length: reductions still in flight are waited for.
  uint32_t h1[16];
  const uint4* g4 = reinterpret_cast<const uint4*>(g_hist) + tid * 4;
  const uint64_t t_h = global_timer_ns();
  while (true) {
    uint32_t part = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint4 v = tid < kFH1Threads ? __ldcg(g4 + k) : make_uint4(0u, 0u, 0u, 0u);
      h1[4 * k] = v.x; h1[4 * k + 1] = v.y; h1[4 * k + 2] = v.z; h1[4 * k + 3] = v.w;
      part += v.x + v.y + v.z + v.w;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
    if (lane == 0) s.sc.warp_tot[warp] = static_cast<int>(part);
    __syncthreads();
    if (tid == 0) {
      uint32_t t = 0;
      for (int w = 0; w < kFThreads / 32; ++w) t += static_cast<uint32_t>(s.sc.warp_tot[w]);
      const bool complete = t == static_cast<uint32_t>(L);
      const bool timeout = !complete && global_timer_ns() - t_h > kWaitTimeoutNs;
      if (timeout) report(p.ws, DSAI_STATUS_WAIT_TIMEOUT);
      s.hist_done = (complete || timeout) ? 1 : 0;
    }
    __syncthreads();
    if (s.hist_done) break;
    __nanosleep(256);
  }

  if (tid == 0) s.extreme[0] = h1[0] != 0u;
  if (tid == kFH1Threads - 1) {
    uint32_t x = 0u;
#pragma unroll
    for (int i = 8; i < 16; ++i) x |= h1[i];
    s.extreme[1] = x != 0u;
  }
  find_threshold<kFThreads, 16>(s.sc, h1, kTopK);  // its barriers publish the zeroed counters
  if (tid < kFH1Threads) {
    uint4* gz = reinterpret_cast<uint4*>(g_hist) + tid * 4;
#pragma unroll
    for (int k = 0; k < 4; ++k) __stcg(gz + k, make_uint4(0u, 0u, 0u, 0u));  // clean for the next call
  }
  if (tid == 0) g_hist[kRowDone] = 0u;
  const uint32_t bin1 = static_cast<uint32_t>(s.sc.sel_bin);
  const int above1 = s.sc.sel_above;
  const int n1 = s.sc.sel_count;
  const bool listed = n1 <= kFCap;
  const uint32_t key_lo = bin1 << (32 - kHistBits);
  const uint32_t key_top = key_lo | ((1u << (32 - kHistBits)) - 1u);
  const int k1 = kTopK - above1;
  const bool fast_skip = (s.extreme[0] | s.extreme[1]) == 0;
  const float f_lo = key_to_float(key_lo);

  auto value_of = [&](int i) -> int32_t {
    const int32_t page = bt_cached ? s.bt[i >> 6] : bt_row[i >> 6];
    return page * kPage + (i & (kPage - 1));
  };

  bool landed = true;
  for (int r = 0; r < nrounds; ++r) {
    const int base = r * kFRound;
    float4(*vals)[kFThreads] = s.vals[r % kFRing];
    cp_async_wait_group<kFRing - 1>();  // this thread's copies of round r have landed
    uint32_t gtm = 0u, inm = 0u;
    const int groups = min(kFPer / 4, (L - base + 4 * kFThreads - 1) / (4 * kFThreads));
#pragma unroll
    for (int u = 0; u < kFPer / 4; ++u) {
      if (u < groups) {
        const int left = L - (base + 4 * (u * kFThreads + tid));
        const uint32_t valid = left >= 4 ? 0xFu : (left > 0 ? (1u << left) - 1u : 0u);
        float4 w = vals[u][tid];
        if (valid) {
          if (!settle(w, row + base + 4 * (u * kFThreads + tid), valid)) landed = false;
          vals[u][tid] = w;
        }
        if (fast_skip && fmaxf(fmaxf(w.x, w.y), fmaxf(w.z, w.w)) < f_lo) continue;
        const uint32_t k4[4] = {key_of_bits(__float_as_uint(w.x)), key_of_bits(__float_as_uint(w.y)),
                                key_of_bits(__float_as_uint(w.z)), key_of_bits(__float_as_uint(w.w))};
        uint32_t g = 0u, n = 0u;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          g |= static_cast<uint32_t>(k4[c] > key_top) << c;
          n |= static_cast<uint32_t>(k4[c] >= key_lo) << c;
        }
        g &= valid;
        n &= valid;
        gtm |= g << (4 * u);
        inm |= n << (4 * u);
      }
    }
    const uint32_t eqm = listed ? (inm & ~gtm) : 0u;
    int pos = warp_alloc_n(&s.out_count, __popc(gtm));
    int cpos = warp_alloc_n(&s.cand_count, __popc(eqm));
    auto entry = [&](int e) { return base + 4 * ((e >> 2) * kFThreads + tid) + (e & 3); };
    auto key_of_entry = [&](int e) {
      return key_of_bits(__float_as_uint(reinterpret_cast<const float*>(&vals[e >> 2][tid])[e & 3]));
    };
    for (uint32_t m = gtm; m; m &= m - 1u) {  // above the pivot bin: straight to the output
      const int e = __ffs(m) - 1;
      out.emit(pos++, value_of(entry(e)), 0u);
    }
    for (uint32_t m = eqm; m; m &= m - 1u) {  // in the pivot bin: to the list
      const int e = __ffs(m) - 1;
      const uint32_t key = key_of_entry(e);
      if (cpos < kFCap) {
        s.cand_key[cpos] = key;
        s.cand_val[cpos] = value_of(entry(e));
      }
      ++cpos;
      atomicAdd(&s.hist[(key >> 10) & (kBins2 - 1)], 1u);
    }
    load_round(r + kFRing);  // refill this slot (this thread's entries only)
  }
  cp_async_wait_group<0>();
  if (!landed) report(p.ws, DSAI_STATUS_WAIT_TIMEOUT);
  __syncthreads();  // candidates, second-digit counts and output slots are final

  if (!listed) {
    // More keys in the pivot bin than the list holds: the second digit over
    // the row in global memory (every entry has landed by now).
    for (int base = 0; base < L; base += kFThreads) {
      const int i = base + tid;
      const uint32_t key = i < L ? ordered_key(__ldcg(row + i)) : 0u;
      hist_add(s.hist, (key >> 10) & (kBins2 - 1), i < L && (key >> (32 - kHistBits)) == bin1);
    }
    __syncthreads();
  }
  uint32_t h2[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) h2[i] = tid < kFH2Threads ? s.hist[4 * tid + i] : 0u;
  find_threshold<kFThreads, 4>(s.sc, h2, k1);
  const uint32_t prefix2 = (bin1 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
  const int k2 = k1 - s.sc.sel_above;  // keys still needed from the second-digit bin
  const int n2 = s.sc.sel_count;
  const bool small = n2 <= kFSmall;

  const int n3 = listed ? min(s.cand_count, kFCap) : L;
  auto key_at = [&](int j) -> uint32_t {
    if (listed) return s.cand_key[j];
    const uint32_t key = ordered_key(__ldcg(row + j));
    return (key >> (32 - kHistBits)) == bin1 ? key : 0u;
  };
  auto val_at = [&](int j) -> int32_t {
    if (listed) return s.cand_val[j];
    return physical_id(bt_row, j);
  };

  if (small) {
    for (int base = 0; base < n3; base += kFThreads) {
      const int j = base + tid;
      const uint32_t key = j < n3 ? key_at(j) : 0u;
      const bool in = j < n3 && key != 0u && (key >> (32 - kHistBits)) == bin1;
      const bool gt = in && (key >> 10) > prefix2;
      const bool eq = in && (key >> 10) == prefix2;
      const int pos = warp_alloc_1(&s.out_count, gt);
      const int q = warp_alloc_1(&s.small_count, eq);
      if (gt) out.emit(pos, val_at(j), key);
      if (eq && q < kFSmall) {
        s.small_key[q] = key;
        s.small_val[q] = val_at(j);
      }
    }
    __syncthreads();
    const int n = min(s.small_count, kFSmall);
    if (tid < n) {
      const uint32_t ki = s.small_key[tid];
      int r = 0;
      for (int j = 0; j < n; ++j) {
        const uint32_t kj = s.small_key[j];
        r += (kj > ki || (kj == ki && j < tid)) ? 1 : 0;
      }
      if (r < k2) out.emit(kTopK - k2 + r, s.small_val[tid], ki);
    }
  } else {
    // Many keys share the 22-bit prefix: count the third digit over them.
    for (int i = tid; i < kBins2; i += kFThreads) s.hist[i] = 0u;
    __syncthreads();
    for (int base = 0; base < n3; base += kFThreads) {
      const int j = base + tid;
      const uint32_t key = j < n3 ? key_at(j) : 0u;
      if (j < n3 && key != 0u && (key >> 10) == prefix2) atomicAdd(&s.hist[key & (kBins2 - 1)], 1u);
    }
    __syncthreads();
    uint32_t h3[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) h3[i] = tid < kFH2Threads ? s.hist[4 * tid + i] : 0u;
    find_threshold<kFThreads, 4>(s.sc, h3, k2);
    const uint32_t pivot = (prefix2 << 10) | static_cast<uint32_t>(s.sc.sel_bin);
    const int k3 = k2 - s.sc.sel_above;  // how many keys equal to the pivot are taken
    for (int base = 0; base < n3; base += kFThreads) {
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
  __syncthreads();  // every read of the row's logits is done
  if (!p.keep_logits) {
    // The sentinel back over the row's logits, for the next call.
    const float4 sent = make_float4(__uint_as_float(kSentinel), __uint_as_float(kSentinel),
                                    __uint_as_float(kSentinel), __uint_as_float(kSentinel));
    float4* r4 = reinterpret_cast<float4*>(row);
    for (int i = tid; i < (L + 3) / 4; i += kFThreads) __stcg(r4 + i, sent);
  }
}

__device__ void selector_role(FusedSmem& sm, const FusedParams& p, int sel, int nsel) {
  SelectorSmem& s = sm.u.se;
  const int tid = threadIdx.x;
  // Rows that fit in the top-K: every token in order, -1 padding
  // (reference kernel.cu:897-905), spread over the selectors.
  for (int b = sel; b < p.rows; b += nsel) {
    const int L = row_len(p.seq_lens, b, p.max_pages, nullptr);
    if (L > kTopK) continue;
    const int32_t* bt_row = p.block_table + static_cast<size_t>(b) * p.max_pages;
    int32_t* o = p.out_ids + static_cast<size_t>(b) * kTopK;
    for (int i = tid; i < kTopK; i += kFThreads) o[i] = i < L ? physical_id(bt_row, i) : -1;
  }
  // The other rows, in the order they are scored: take a position, wait for
  // its row's tiles, select.
  while (true) {
    if (tid == 0) {
      int item = -1;
      while (true) {
        const int k = atomicAdd(p.ws + kCtlHead, 1);
        if (k >= p.rows) break;
        const int b = sm.order[k];
        if (row_len(p.seq_lens, b, p.max_pages, nullptr) <= kTopK) continue;  // written above
        const uint32_t total = 4u * static_cast<uint32_t>(sm.row_start[k + 1] - sm.row_start[k]);
        const uint32_t* done = p.hist + static_cast<size_t>(b) * kHistStride + kRowDone;
        uint32_t v = ld_relaxed_gpu(done);
        if (v != total) {
          const uint64_t t0 = global_timer_ns();
          uint32_t n = 0;
          while ((v = ld_relaxed_gpu(done)) != total) {
            __nanosleep(128);
            if ((++n & 15u) == 0u && global_timer_ns() - t0 > kWaitTimeoutNs) break;
          }
        }
        if (v == total) {
          item = b;
        } else {
          report(p.ws, DSAI_STATUS_WAIT_TIMEOUT);
        }
        break;
      }
      s.item = item;
    }
    __syncthreads();
    const int b = s.item;
    if (b < 0) break;
    select_row(s, p, b);
    __syncthreads();
  }
  if (tid == 0) {
    // The last selector to leave resets the claim counter for the next call:
    // every selector has taken its last position.
    const int f = atomicAdd(p.ws + kCtlFin, 1);
    if (f == nsel - 1) {
      atomicExch(p.ws + kCtlHead, 0);
      atomicExch(p.ws + kCtlFin, 0);
    }
  }
}

__global__ void __launch_bounds__(kFThreads, 1)
    fused_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                 const __grid_constant__ CUtensorMap tmap_s, const FusedParams p) {
  extern __shared__ uint8_t smem_raw[];
  FusedSmem& sm = *reinterpret_cast<FusedSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool scorer = static_cast<int>(blockIdx.x) < p.scorers;
  const int pipe = warp / kFPipeWarps;

  // Shared memory and kernel parameters only before the programmatic wait.
  if (scorer && (warp % kFPipeWarps) == 0 && lane == 0) {
    PipeSmem& s = sm.u.pipe[pipe];
    for (int i = 0; i < kFStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < kFScaleSlots; ++i) {
      mbar_init(&s.sfull[i], 1);
      mbar_init(&s.sempty[i], kFEpiWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.qfull[i], 1);
      mbar_init(&s.qempty[i], 1 + kFEpiWarps);  // MMA commit + every epilogue warp
    }
    for (int i = 0; i < kFAccs; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], kFEpiWarps);
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_mbar_init();
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_s);
  }
  grid_dep_wait();
  grid_dep_launch_dependents();
  build_order(sm, p);
  if (!scorer) {
    selector_role(sm, p, static_cast<int>(blockIdx.x) - p.scorers, static_cast<int>(gridDim.x) - p.scorers);
    return;
  }
  if (warp == 1) {
    tmem_alloc(&sm.tmem_base, kFTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pipe_role(sm, sm.u.pipe[pipe], sm.tmem_base + static_cast<uint32_t>(pipe * kFPipeTmemCols), &tmap_q, &tmap_k,
            &tmap_s, p, static_cast<int>(blockIdx.x) * kFPipes + pipe, p.scorers * kFPipes);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(sm.tmem_base, kFTmemCols);
  }
}

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  if (!v || !*v) return dflt;
  return atoi(v);
}

}  // namespace

bool fused_enabled() {
  static const int on = env_int("DSAI_FUSED", 0);
  return on != 0;
}

uint32_t fused_logits_sentinel() { return kSentinel; }

cudaError_t launch_fused(const FusedLaunch& lp, const CUtensorMap& tmap_q, const CUtensorMap& tmap_k,
                         const CUtensorMap& tmap_s, cudaStream_t stream) {
  static bool attr_set[64] = {};  // the attributes are per function and device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kFSmemBytes);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  // One CTA per SM.  Selectors only wait for scorers and scorers never wait
  // for selectors, so the grid completes even if fewer CTAs were resident
  // at once.
  const int grid = lp.sms;
  static const int sel_env = env_int("DSAI_FUSED_SELECTORS", 0);
  static const int chunk_env = env_int("DSAI_FUSED_CHUNK", 0);
  int nsel = sel_env > 0 ? sel_env : lp.rows / 4;
  nsel = nsel < 4 ? 4 : (nsel > 32 ? 32 : nsel);
  if (nsel > grid / 4) nsel = grid / 4;
  FusedParams p;
  p.weights = lp.weights;
  p.seq_lens = lp.seq_lens;
  p.block_table = lp.block_table;
  p.logits = lp.logits;
  p.hist = lp.hist;
  p.ws = lp.ws;
  p.out_ids = lp.out_ids;
  p.rows = lp.rows;
  p.max_pages = lp.max_pages;
  p.num_pages = lp.num_pages;
  p.ld = lp.ld;
  p.score_all = lp.score_all;
  p.keep_logits = lp.keep_logits;
  p.scorers = grid - nsel;
  p.chunk = chunk_env > 0 ? chunk_env : 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(kFThreads);
  cfg.dynamicSmemBytes = kFSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fused_kernel, tmap_q, tmap_k, tmap_s, p);
}

}  // namespace dsai
