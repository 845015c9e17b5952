// score.cu — paged FP8 scoring of the index-K cache on tcgen05 tensor cores.
//
// For every scored row b and token t < L_b it writes the fp32 logit
//   logit[b,t] = scale[page,slot] * sum_h ReLU(sum_d q[b,h,d] K[page,slot,d]) * w[b,h]
// (the math of the reference's stage 1, solution/python/kernel.cu:5-9 and
// :811-831, kept in fp32 instead of the reference's fp16 store), and the
// per-row histogram of the logits' top 12 ordered-key bits that the
// selection kernel starts from.
//
// Work decomposition.  A row of L tokens is cut into ceil(L/128) tiles of two
// 64-token pages (M = 128 of one UMMA).  All tiles of all scored rows form
// one flat sequence of T tiles.  Its first part (T - D tiles) is cut into
// contiguous static slices, one per CTA of the persistent grid; its last D
// tiles are dealt out in chunks of `chunk` tiles that CTAs claim with one
// atomic on a counter in the workspace header as they run out of work, so
// CTAs that start late (their SM still held by the previous kernel) or run
// slow take fewer tiles and the grid ends together.  The producer hands each
// chunk's tile range to the MMA and epilogue warps through a small shared-
// memory ring; the last producer to run out of chunks resets the counters
// for the next launch.  Q is reloaded only at row changes.
//
// Two CTAs per SM (two independent pipelines per SM overlap each other's
// latencies), 6 warps each, warp-specialised:
//   warp 0      producer: follows block_table and TMA-loads each page (8 KB,
//               128-B swizzle) into a 5-stage K ring, its 64 scales into a
//               16-slot scale ring, and the row's Q (8 KB) into a 2-slot ring.
//               The 32 lanes resolve the pages of 32 tiles at once, one batch
//               ahead within a chunk.
//   warp 1      MMA issuer (one lane): 4 x tcgen05.mma kind::f8f6f4
//               M128 N64 K32 per tile into one of 4 TMEM accumulators.  A K
//               stage is released as soon as its MMAs complete.
//   warps 2-5   epilogue: tcgen05.ld of the 128x64 fp32 tile (one token per
//               thread, 64 head scores in registers), ReLU, head weights,
//               token scale, coalesced fp32 store, and fire-and-forget
//               reductions into the row's global histogram of 12-bit key
//               prefixes, one per distinct bin of the warp's 32 tokens (no
//               group synchronisation beyond the warp, so a timed-out warp
//               can never leave the others waiting).
// Rows with L <= 2048 are skipped (their output does not depend on scores).
#include <cstdlib>

#include "common.cuh"
#include "graph.h"
#include "launch.h"
#include "sm100.cuh"
#include "tiles.cuh"

namespace dsai {
namespace {

using namespace sm100;

constexpr int kCtasPerSm = 2;                  // two independent pipelines per SM
constexpr int kStages = 5;
constexpr int kScaleSlots = 16;
constexpr int kAccs = 4;
constexpr int kAccCols = kHeads;               // 64 fp32 columns per accumulator
constexpr int kTmemCols = kAccs * kAccCols;    // 256 (power of two >= 32)
constexpr int kThreads = 192;
constexpr int kEpiThreads = 128;
constexpr uint32_t kScaleTx = kPage * 4;       // 256 B of scales per page

struct ScoreParams {
  const float* weights;
  const int32_t* seq_lens;
  const int32_t* block_table;
  float* logits;
  uint32_t* hist;     // [rows, kHistStride] (rows of this launch)
  int* status;
  int rows;
  int max_pages;
  int num_pages;
  int ld;
  int row_base;
  int score_all;
  int dyn_pct;        // percent of the tile sequence dealt out in chunks (0: static slices only) ...
  int dyn_per_cta;    // ... but at most this many tiles per CTA of the grid
  int chunk;          // tiles per claimed chunk
};

constexpr int kChunkSlots = 4;  // chunk ranges in flight from the producer to the consumers
constexpr int kDynPercent = 25;  // default share of the tile sequence dealt out in chunks,
constexpr int kDynPerCta = 8;    // capped at this many tiles per CTA
constexpr int kDynChunk = 4;     // default tiles per chunk
constexpr int kDynMinPerCta = 8; // chunks only when the sequence has this many tiles per CTA

int env_int_or(const char* name, int dflt) {
  const char* v = getenv(name);
  return (v && *v) ? atoi(v) : dflt;
}

struct ScoreSmem {
  uint8_t k[kStages][2 * kPageKBytes];  // 1024-B aligned stages, SW128 K-major
  uint8_t q[2][kQBytes];                // SW128 K-major, N = 64 heads
  float scale[kScaleSlots][kTileTok];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t sfull[kScaleSlots];
  uint64_t sempty[kScaleSlots];
  uint64_t qfull[2];
  uint64_t qempty[2];
  uint64_t tfull[kAccs];
  uint64_t tempty[kAccs];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int warp_sums[kThreads / 32];
  int row_start[kMaxRowsPerLaunch + 1];
  // Chunked kernel only: the ring of chunk ranges [x, y) (x < 0: no more work).
  uint64_t cfull[kChunkSlots];
  uint64_t cempty[kChunkSlots];
  int2 chunk[kChunkSlots];
};

constexpr int kSmemBytes = static_cast<int>(sizeof(ScoreSmem)) + 1024;
static_assert(kCtasPerSm * (kSmemBytes + 1024) <= 233472, "two CTAs per SM must fit");

__device__ __forceinline__ void fail(ScoreSmem& s, int* status) {
  report(status, DSAI_STATUS_WAIT_TIMEOUT);
  *reinterpret_cast<volatile int*>(&s.abort) = 1;
}

// Exclusive scan of per-row tile counts into s.row_start (all threads).
__device__ void build_row_table(ScoreSmem& s, const ScoreParams& p) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (p.rows + kThreads - 1) / kThreads;
  const int b0 = min(p.rows, tid * per), b1 = min(p.rows, b0 + per);
  int* st = blockIdx.x == 0 ? p.status : nullptr;
  int sum = 0;
  for (int b = b0; b < b1; ++b)
    sum += row_tiles(row_len(p.seq_lens, b, p.max_pages, st), p.score_all != 0);
  int incl = sum;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) s.warp_sums[warp] = incl;
  __syncthreads();
  int warp_excl = 0;
  for (int w = 0; w < warp; ++w) warp_excl += s.warp_sums[w];
  int prefix = warp_excl + incl - sum;
  for (int b = b0; b < b1; ++b) {
    s.row_start[b] = prefix;
    prefix += row_tiles(row_len(p.seq_lens, b, p.max_pages, nullptr), p.score_all != 0);
  }
  if (tid == kThreads - 1) s.row_start[p.rows] = prefix;
}

// Page ids of one tile, resolved by one producer lane.
struct TileRef {
  int row, pg0, pg1, two;
};

__device__ __forceinline__ TileRef resolve_tile(const ScoreSmem& s, const ScoreParams& p, int t) {
  TileRef r;
  r.row = find_row(s.row_start, p.rows, t);
  const int j = t - s.row_start[r.row];
  const int32_t* bt = p.block_table + static_cast<size_t>(r.row) * p.max_pages;
  // The second page is read unconditionally when it is inside the row of the
  // block table (in bounds); it is used only when the row reaches it.
  const int L = row_len(p.seq_lens, r.row, p.max_pages, nullptr);
  r.pg0 = bt[2 * j];
  r.pg1 = (2 * j + 1 < p.max_pages) ? bt[2 * j + 1] : 0;
  r.two = (2 * j + 1) * kPage < L;
  return r;
}

// Position in the ring of chunk ranges (slot and phase parity).
struct ChunkRing {
  int slot = 0;
  uint32_t phase = 0;
};

// kChunked: the tail of the sequence dealt out in chunks (see the top of the
// file); without it every CTA takes one static slice and none of the chunk
// machinery (ring barriers, counters) is compiled in: small launches, where
// that machinery's set-up sits on the critical path, use this form.
template <bool kChunked>
__global__ void __launch_bounds__(kThreads, kCtasPerSm)
    score_kernel(const __grid_constant__ CUtensorMap tmap_q,
                 const __grid_constant__ CUtensorMap tmap_k,
                 const __grid_constant__ CUtensorMap tmap_s, const ScoreParams p) {
  extern __shared__ uint8_t smem_raw[];
  ScoreSmem& s = *reinterpret_cast<ScoreSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // Launched as a programmatic dependent: the barriers and the tensor-map
  // prefetch (shared memory and kernel parameters only) overlap the previous
  // kernel's tail; global memory is touched only after the wait.  (TMEM is
  // allocated after it: a predecessor still running on this SM may need it.)
  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);                 // MMA commit
    }
    for (int i = 0; i < kScaleSlots; ++i) {
      mbar_init(&s.sfull[i], 1);
      mbar_init(&s.sempty[i], kEpiThreads / 32);  // 4 epilogue warps
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.qfull[i], 1);
      mbar_init(&s.qempty[i], 1);
    }
    for (int i = 0; i < kAccs; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], kEpiThreads / 32);
    }
    if constexpr (kChunked) {
      for (int i = 0; i < kChunkSlots; ++i) {
        mbar_init(&s.cfull[i], 1);
        mbar_init(&s.cempty[i], 1 + kEpiThreads / 32);  // the MMA issuer + the epilogue warps
      }
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmap_q);
    prefetch_tmap(&tmap_k);
    prefetch_tmap(&tmap_s);
  }
  sm100::grid_dep_wait();
  sm100::grid_dep_launch_dependents();
  build_row_table(s, p);
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const int* rs = s.row_start;
  const int T = rs[p.rows];
  // Tiles dealt out in chunks: enough to absorb CTAs that start late or run
  // slow (a few tiles each), not a share that grows with the sequence; none
  // when the grid has few tiles per CTA (a chunk would then put several
  // tiles on one CTA that the static slices spread over several).
  const bool dyn = kChunked && T >= static_cast<int>(gridDim.x) * kDynMinPerCta;
  const int D = dyn ? static_cast<int>(min(static_cast<long long>(T) * min(100, max(0, p.dyn_pct)) / 100,
                                           static_cast<long long>(gridDim.x) * max(0, p.dyn_per_cta)))
                    : 0;
  const int TS = T - D;                           // tiles in static slices
  const int C = max(1, p.chunk);
  const int nchunks = (D + C - 1) / C;
  const int t0 = static_cast<int>((static_cast<long long>(TS) * blockIdx.x) / gridDim.x);
  const int t1 = static_cast<int>((static_cast<long long>(TS) * (blockIdx.x + 1)) / gridDim.x);
  int* const claim_ctr = p.status + kHdrScoreNext;
  // Chunk ranges go through the shared-memory ring only when chunks exist;
  // otherwise every role walks its static slice directly.
  const bool use_ring = kChunked && nchunks > 0;

  if (!use_ring && t0 >= t1) {
    // No tiles for this CTA and none to claim (small grids leave most CTAs idle).
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_k = l2_policy_evict_first();
    const uint64_t pol_q = l2_policy_evict_last();
    int stage = 0, sslot = 0, qs = 1, cur_row = -1;
    uint32_t phase = 0, sphase = 0;
    uint32_t qe_par[2] = {0u, 0u};
    int q_uses[2] = {0, 0};
    int k_fills = 0, s_fills = 0;
    ChunkRing ring;
    bool ok = true;
    bool claims_left = nchunks > 0;
    int cb = t0, ce = t1;  // the static slice first
    while (ok) {
      if (use_ring) {
        // Publish [cb, ce) (cb < 0: no more work) to the MMA issuer and the epilogue.
        int good = 1;
        if (lane == 0) {
          if (!mbar_wait(&s.cempty[ring.slot], ring.phase ^ 1u, &s.abort, kWaitTimeoutNs)) {
            good = 0;
            fail(s, p.status);
          } else {
            s.chunk[ring.slot] = make_int2(cb, ce);
            mbar_arrive(&s.cfull[ring.slot]);
          }
        }
        if (++ring.slot == kChunkSlots) { ring.slot = 0; ring.phase ^= 1u; }
        good = __shfl_sync(0xffffffffu, good, 0);
        if (!good) break;
      }
      if (cb < 0) break;

      TileRef nxt = {0, 0, 0, 0};
      if (cb + lane < ce) nxt = resolve_tile(s, p, cb + lane);
      for (int tb = cb; tb < ce && ok; tb += 32) {
        const TileRef cur = nxt;
        // Resolve the chunk's next batch now; its loads overlap this batch's issue.
        if (tb + 32 + lane < ce) nxt = resolve_tile(s, p, tb + 32 + lane);
        if (tb + lane < ce &&
            (static_cast<unsigned>(cur.pg0) >= static_cast<unsigned>(p.num_pages) ||
             (cur.two && static_cast<unsigned>(cur.pg1) >= static_cast<unsigned>(p.num_pages))))
          report(p.status, DSAI_STATUS_BAD_PAGE);  // TMA zero-fills out-of-range pages
        const int n = min(32, ce - tb);
        for (int i = 0; i < n; ++i) {
          const int r = __shfl_sync(0xffffffffu, cur.row, i);
          const int a = __shfl_sync(0xffffffffu, cur.pg0, i);
          const int b = __shfl_sync(0xffffffffu, cur.pg1, i);
          const int tw = __shfl_sync(0xffffffffu, cur.two, i);
          int g = 1;
          if (lane == 0) {
            if (r != cur_row) {
              cur_row = r;
              qs ^= 1;
              // The slot is free once the MMAs of its last row completed.
              if (!mbar_wait(&s.qempty[qs], qe_par[qs] ^ 1u, &s.abort, kWaitTimeoutNs)) {
                g = 0;
              } else {
                qe_par[qs] ^= 1u;
                ++q_uses[qs];
                mbar_arrive_expect_tx(&s.qfull[qs], kQBytes);
                tma_load_2d(s.q[qs], &tmap_q, &s.qfull[qs], 0, (p.row_base + r) * kHeads, pol_q);
              }
            }
            if (g && !mbar_wait(&s.empty[stage], phase ^ 1u, &s.abort, kWaitTimeoutNs)) g = 0;
            if (g && !mbar_wait(&s.sempty[sslot], sphase ^ 1u, &s.abort, kWaitTimeoutNs)) g = 0;
            if (g) {
              mbar_arrive_expect_tx(&s.full[stage], tw ? 2 * kPageKBytes : kPageKBytes);
              mbar_arrive_expect_tx(&s.sfull[sslot], tw ? 2 * kScaleTx : kScaleTx);
              tma_load_3d(s.k[stage], &tmap_k, &s.full[stage], 0, 0, a, pol_k);
              tma_load_2d(s.scale[sslot], &tmap_s, &s.sfull[sslot], 0, a, pol_k);
              if (tw) {
                tma_load_3d(s.k[stage] + kPageKBytes, &tmap_k, &s.full[stage], 0, 0, b, pol_k);
                tma_load_2d(s.scale[sslot] + kPage, &tmap_s, &s.sfull[sslot], 0, b, pol_k);
              }
              ++k_fills;
              ++s_fills;
              if (++stage == kStages) { stage = 0; phase ^= 1u; }
              if (++sslot == kScaleSlots) { sslot = 0; sphase ^= 1u; }
            } else {
              fail(s, p.status);
            }
          }
          g = __shfl_sync(0xffffffffu, g, 0);
          if (!g) { ok = false; break; }
        }
      }
      if (!use_ring) break;  // the static slice was all there is
      // The next chunk, claimed only now that this one's tiles are all
      // issued: the K ring still holds several tiles for the consumers, which
      // covers the claim's latency, and no CTA sits on a chunk it has not
      // started while others run dry at the end.
      int nb = -1, ne = -1;
      if (lane == 0 && ok && claims_left) {
        const int k = atomicAdd(claim_ctr, 1);
        if (k < nchunks) {
          nb = TS + k * C;
          ne = min(T, nb + C);
        } else {
          claims_left = false;
        }
      }
      cb = __shfl_sync(0xffffffffu, nb, 0);
      ce = __shfl_sync(0xffffffffu, ne, 0);
    }
    // This producer makes no more claims.  The last one of the grid to get
    // here resets both counters for the next launch on this workspace (which
    // starts only after this grid has completed): off the consumers' path,
    // which still drain the last tiles.
    if (kChunked && lane == 0 && nchunks > 0 &&
        atomicAdd(p.status + kHdrScoreDone, 1) == static_cast<int>(gridDim.x) - 1) {
      *reinterpret_cast<volatile int*>(claim_ctr) = 0;
      *reinterpret_cast<volatile int*>(p.status + kHdrScoreDone) = 0;
    }
    // Never leave with a TMA in flight: wait for the latest fill of every
    // slot (each earlier fill of a slot was consumed, hence complete).
    if (lane == 0) {
      for (int i = 0; i < kStages && i < k_fills; ++i) {
        const int last = k_fills - 1 - i;  // fill index of the i-th latest fill
        if (!mbar_wait(&s.full[last % kStages], (last / kStages) & 1, nullptr, kWaitTimeoutNs))
          report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
      }
      for (int i = 0; i < kScaleSlots && i < s_fills; ++i) {
        const int last = s_fills - 1 - i;
        if (!mbar_wait(&s.sfull[last % kScaleSlots], (last / kScaleSlots) & 1, nullptr, kWaitTimeoutNs))
          report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
      }
      for (int i = 0; i < 2; ++i)
        if (q_uses[i] > 0 && !mbar_wait(&s.qfull[i], (q_uses[i] - 1) & 1, nullptr, kWaitTimeoutNs))
          report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_e4m3_f32(kTileTok, kHeads);
      int stage = 0, acc = 0, qs = 1, cur_row = -1;
      uint32_t phase = 0, aphase = 0;
      uint32_t qf_par[2] = {0u, 0u};
      ChunkRing ring;
      bool ok = true;
      bool more = true;  // without the ring: the static slice, once
      while (ok && more) {
        int2 ch = make_int2(t0, t1);
        if (use_ring) {
          if (!mbar_wait(&s.cfull[ring.slot], ring.phase, &s.abort, kWaitTimeoutNs)) { fail(s, p.status); break; }
          ch = s.chunk[ring.slot];
          mbar_arrive(&s.cempty[ring.slot]);
          if (++ring.slot == kChunkSlots) { ring.slot = 0; ring.phase ^= 1u; }
        } else {
          more = false;
        }
        if (ch.x < 0) break;
        if (ch.x >= ch.y) continue;
        Cursor c;
        c.init(rs, p.rows, ch.x);
        for (; c.t < ch.y; c.next(rs, ch.y)) {
          if (c.row != cur_row) {
            if (cur_row >= 0) umma_commit(&s.qempty[qs]);  // previous row's Q free when done
            cur_row = c.row;
            qs ^= 1;
            if (!mbar_wait(&s.qfull[qs], qf_par[qs], &s.abort, kWaitTimeoutNs)) { fail(s, p.status); ok = false; break; }
            qf_par[qs] ^= 1u;
          }
          if (!mbar_wait(&s.full[stage], phase, &s.abort, kWaitTimeoutNs)) { fail(s, p.status); ok = false; break; }
          if (!mbar_wait(&s.tempty[acc], aphase ^ 1u, &s.abort, kWaitTimeoutNs)) { fail(s, p.status); ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(s.k[stage]));
          const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(s.q[qs]));
          const uint32_t d = s.tmem_base + static_cast<uint32_t>(acc * kAccCols);
#pragma unroll
          for (int kk = 0; kk < kDim / 32; ++kk)  // K = 32 e4m3 (32 B) per MMA
            umma_f8(d, adesc + 2u * kk, bdesc + 2u * kk, idesc, kk > 0 ? 1u : 0u);
          umma_commit(&s.empty[stage]);  // K stage free once these MMAs are done
          umma_commit(&s.tfull[acc]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
          if (++acc == kAccs) { acc = 0; aphase ^= 1u; }
        }
      }
      // Every MMA issued by this thread has completed once this arrives.
      umma_commit(&s.drain);
      if (!mbar_wait(&s.drain, 0, nullptr, kWaitTimeoutNs)) report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;              // TMEM lanes [32*quad, 32*quad+32)
    const int tok = quad * 32 + lane;       // token of the tile owned by this thread
    int acc = 0, sslot = 0, cur_row = -1, L = 0;
    uint32_t aphase = 0, sphase = 0;
    bool hist_row = false;
    float w[kHeads];
    float* out_row = nullptr;
    uint32_t* hist_g = nullptr;
    ChunkRing ring;
    bool ok = true;
    bool more = true;  // without the ring: the static slice, once
    while (ok && more) {
      int2 ch = make_int2(t0, t1);
      if (use_ring) {
        // Waits are decided warp-wide: the warp runs warp-collective steps below.
        if (!__all_sync(0xffffffffu, mbar_wait(&s.cfull[ring.slot], ring.phase, &s.abort, kWaitTimeoutNs))) {
          fail(s, p.status);
          break;
        }
        ch = s.chunk[ring.slot];
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.cempty[ring.slot]);
        if (++ring.slot == kChunkSlots) { ring.slot = 0; ring.phase ^= 1u; }
      } else {
        more = false;
      }
      if (ch.x < 0) break;
      if (ch.x >= ch.y) continue;
      Cursor c;
      c.init(rs, p.rows, ch.x);
      for (; c.t < ch.y; c.next(rs, ch.y)) {
        if (c.row != cur_row) {
          cur_row = c.row;
          // (Staging the weights in shared memory with the row's Q instead
          // made the kernel ~1.8 us slower: the epilogue then waits for Q.)
          const float4* w4 = reinterpret_cast<const float4*>(p.weights + static_cast<size_t>(cur_row) * kHeads);
#pragma unroll
          for (int i = 0; i < kHeads / 4; ++i) {
            const float4 v = __ldg(w4 + i);
            w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
          }
          L = row_len(p.seq_lens, cur_row, p.max_pages, nullptr);
          hist_row = L > kTopK;  // only rows that go through the radix select
          out_row = p.logits + static_cast<size_t>(cur_row) * p.ld;
          hist_g = p.hist + static_cast<size_t>(cur_row) * kHistStride;
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&s.tfull[acc], aphase, &s.abort, kWaitTimeoutNs))) {
          fail(s, p.status);
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r0[32], r1[32];
        const uint32_t taddr = s.tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                               static_cast<uint32_t>(acc * kAccCols);
        tmem_ld_32x32b_x32(taddr, r0);
        tmem_ld_32x32b_x32(taddr + 32u, r1);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tempty[acc]);
        if (!__all_sync(0xffffffffu, mbar_wait(&s.sfull[sslot], sphase, &s.abort, kWaitTimeoutNs))) {
          fail(s, p.status);
          ok = false;
          break;
        }
        const float sc = s.scale[sslot][tok];
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.sempty[sslot]);
        // Eight running sums: a_c over heads 4i + c, b_c over 32 + 4i + c,
        // then ((a0+b0)+(a1+b1)) + ((a2+b2)+(a3+b3)) (the group scorer's order).
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
        const float logit = (((a0 + b0) + (a1 + b1)) + ((a2 + b2) + (a3 + b3))) * sc;
        const int t_abs = c.j * kTileTok + tok;
        const bool live = t_abs < L;
        if (live) out_row[t_abs] = logit;
        if (hist_row) {
          // A row's logits crowd into few bins: lanes sharing a bin add once,
          // so the row's reductions do not serialise on a few L2 addresses.
          const uint32_t bin = ordered_key(logit) >> (32 - kHistBits);
          const unsigned act = __ballot_sync(0xffffffffu, live);
          if (live) {
            const unsigned peers = __match_any_sync(act, bin);
            if (lane == __ffs(peers) - 1) atomicAdd(hist_g + bin, static_cast<uint32_t>(__popc(peers)));  // RED
          }
        }
        if (++acc == kAccs) { acc = 0; aphase ^= 1u; }
        if (++sslot == kScaleSlots) { sslot = 0; sphase ^= 1u; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(s.tmem_base, kTmemCols);
  }
}

}  // namespace

int score_smem_bytes() { return kSmemBytes; }

cudaError_t launch_score(const ScoreLaunch& lp, const CUtensorMap& tmap_q, const CUtensorMap& tmap_k,
                         const CUtensorMap& tmap_s, cudaStream_t stream) {
  static bool attr_set[64] = {};  // the attribute is per function and device
  int dev = 0;
  cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return e0;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(score_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kSmemBytes);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(score_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  ScoreParams p;
  p.weights = lp.weights;
  p.seq_lens = lp.seq_lens;
  p.block_table = lp.block_table;
  p.logits = lp.logits;
  p.hist = lp.hist;
  p.status = lp.status;
  p.rows = lp.rows;
  p.max_pages = lp.max_pages;
  p.num_pages = lp.num_pages;
  p.ld = lp.ld;
  p.row_base = lp.row_base;
  p.score_all = lp.score_all;
  // The last part of the tile sequence is dealt out in chunks (both values
  // can be overridden from the environment, read once, for measurements).
  static const int dyn_pct = env_int_or("DSAI_SCORE_DYN", kDynPercent);
  static const int dyn_per_cta = env_int_or("DSAI_SCORE_DYN_CTA", kDynPerCta);
  static const int chunk = env_int_or("DSAI_SCORE_CHUNK", kDynChunk);
  p.dyn_pct = dyn_pct;
  p.dyn_per_cta = dyn_per_cta;
  p.chunk = chunk > 0 ? chunk : 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(lp.grid * kCtasPerSm);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // The chunked form only when the launch can hold enough tiles per CTA for
  // chunks to be dealt out (the kernel checks the true count); the tile count
  // is bounded by rows x tiles of a full block-table row.
  const long long tiles_max = static_cast<long long>(lp.rows) * ((static_cast<long long>(lp.max_pages) + 1) / 2);
  const bool chunked = dyn_pct > 0 && dyn_per_cta > 0 &&
                       tiles_max >= static_cast<long long>(cfg.gridDim.x) * kDynMinPerCta;
  return launch_kernel(cfg, chunked ? score_kernel<true> : score_kernel<false>, tmap_q, tmap_k, tmap_s, p);
}

}  // namespace dsai
