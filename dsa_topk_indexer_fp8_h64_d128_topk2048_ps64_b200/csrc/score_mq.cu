// score_mq.cu — scoring of row groups that share one sequence's K pages:
// multi-query decode, next-n (MTP) speculative rows, the causal rows of a
// prefill chunk.  R consecutive rows (R = 2, 3 or 4) form a group that reads
// one block-table row; every staged K tile is multiplied against the group's
// R stacked queries in a single UMMA, so each K byte crosses HBM once per
// group instead of once per row.
//
// Per row b of a group and token t < L_b the logit is the one the per-row
// scorer computes, with the same arithmetic in the same order (bit-identical
// results):
//   logit[b,t] = scale[page,slot] * sum_h ReLU(sum_d q[b,h,d] K[page,slot,d]) * w[b,h]
// (solution/python/kernel.cu:5-9, :811-831).  The group's pages come from the
// block-table row of its longest row; the rows of a group must agree on every
// page their own lengths reach (they do when they belong to one sequence).
//
// Work decomposition: groups of ceil(Lmax/128) tiles (Lmax = the longest row
// of the group), all groups of a launch in one flat tile sequence, one
// contiguous slice per CTA (tiles.cuh).  A group is scored when any of its
// rows is longer than the top-K (or every row is requested).
//
// One CTA per SM, 2 + 4R warps:
//   warp 0      producer: K pages (TMA, 128-B swizzle) into a ring of as many
//               stages as shared memory holds (9-11: the bytes in flight per
//               SM set the HBM rate this kernel reaches),
//               scales into a 16-slot ring, and at a group change the R
//               queries (R x 8 KB, stacked so they form one N = 64*R operand)
//               and the R x 64 head weights (one bulk copy) into 2-slot rings.
//   warp 1      MMA issuer: 4 x tcgen05.mma kind::f8f6f4 M128 N(64R) K32 per
//               tile into one of the TMEM accumulators (512 columns).
//   warps 2..   epilogue: one warp per (TMEM lane quadrant, group row), so
//               4R warps share the issue slots and hide each other's
//               latencies.  Weights are read from shared memory (broadcast),
//               the head sum runs on packed f32x2 FMAs, and each token's
//               logit is stored and reduced into its row's histogram (one
//               reduction per token), with the row's own length.
#include "common.cuh"
#include "graph.h"
#include "launch.h"
#include "sm100.cuh"
#include "tiles.cuh"

namespace dsai {
namespace {

using namespace sm100;

constexpr int kMqMaxThreads = 64 + 128 * 4;
constexpr int kMqScaleSlots = 16;
constexpr int kMqTmemCols = 512;
constexpr uint32_t kMqScaleTx = kPage * 4;

template <int R>
struct MqTraits {
  static constexpr int kN = kHeads * R;                   // UMMA N: the group's heads
  static constexpr int kAccs = kMqTmemCols / kN >= 4 ? 4 : 2;
  static constexpr int kEpiWarps = 4 * R;                 // one per (lane quadrant, row)
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr int kStages = R == 2 ? 11 : (R == 3 ? 10 : 9);  // fill the shared memory
  static constexpr int kMaxGroups = kMaxRowsPerLaunch / R;
  static_assert(R >= 2 && R <= 4, "2 to 4 rows per group");
  static_assert(kAccs * kN <= kMqTmemCols, "accumulators must fit TMEM");
};

struct MqParams {
  const float* weights;
  const int32_t* seq_lens;
  const int32_t* block_table;
  float* logits;
  uint32_t* hist;
  int* status;
  int rows;        // rows of this launch, a multiple of R
  int max_pages;
  int num_pages;
  int ld;
  int row_base;
  int score_all;
};

template <int R>
struct MqSmem {
  uint8_t k[MqTraits<R>::kStages][2 * kPageKBytes];  // 1024-B aligned stages, SW128 K-major
  uint8_t q[2][R * kQBytes];              // R stacked queries, SW128 K-major, N = 64R
  alignas(128) float w[2][R][kHeads];
  alignas(1024) float scale[kMqScaleSlots][kTileTok];
  uint64_t full[MqTraits<R>::kStages];
  uint64_t empty[MqTraits<R>::kStages];
  uint64_t sfull[kMqScaleSlots];
  uint64_t sempty[kMqScaleSlots];
  uint64_t qfull[2];
  uint64_t qempty[2];
  uint64_t wfull[2];
  uint64_t wempty[2];
  uint64_t tfull[MqTraits<R>::kAccs];
  uint64_t tempty[MqTraits<R>::kAccs];
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
  int warp_sums[kMqMaxThreads / 32];
  int gstart[MqTraits<R>::kMaxGroups + 1];
  int glead[MqTraits<R>::kMaxGroups];  // row (within the launch) whose block-table row the group reads
  int glen[MqTraits<R>::kMaxGroups];   // the group's longest effective row length
};

template <int R>
constexpr int mq_smem_bytes() {
  return static_cast<int>(sizeof(MqSmem<R>)) + 1024;
}
static_assert(mq_smem_bytes<2>() <= 232448 && mq_smem_bytes<3>() <= 232448 && mq_smem_bytes<4>() <= 232448,
              "the group scorer must fit one SM's shared memory");

template <int R>
__device__ __forceinline__ void mq_fail(MqSmem<R>& s, int* status) {
  report(status, DSAI_STATUS_WAIT_TIMEOUT);
  *reinterpret_cast<volatile int*>(&s.abort) = 1;
}

// Per-group longest row, its row index, and the exclusive scan of the group
// tile counts into s.gstart (all threads).
template <int R>
__device__ void build_group_table(MqSmem<R>& s, const MqParams& p) {
  constexpr int kThreads = MqTraits<R>::kThreads;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int groups = p.rows / R;
  const int per = (groups + kThreads - 1) / kThreads;
  const int g0 = min(groups, tid * per), g1 = min(groups, g0 + per);
  int* st = blockIdx.x == 0 ? p.status : nullptr;
  int sum = 0;
  for (int g = g0; g < g1; ++g) {
    int lmax = -1, lead = g * R;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int L = row_len(p.seq_lens, g * R + r, p.max_pages, st);
      if (L > lmax) { lmax = L; lead = g * R + r; }
    }
    s.glen[g] = lmax;
    s.glead[g] = lead;
    sum += row_tiles(lmax, p.score_all != 0);
  }
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
  for (int g = g0; g < g1; ++g) {
    s.gstart[g] = prefix;
    prefix += row_tiles(s.glen[g], p.score_all != 0);
  }
  if (tid == kThreads - 1) s.gstart[groups] = prefix;
}

struct GroupTile {
  int group, pg0, pg1, two;
};

template <int R>
__device__ __forceinline__ GroupTile resolve_group_tile(const MqSmem<R>& s, const MqParams& p, int t) {
  GroupTile r;
  r.group = find_row(s.gstart, p.rows / R, t);
  const int j = t - s.gstart[r.group];
  const int32_t* bt = p.block_table + static_cast<size_t>(s.glead[r.group]) * p.max_pages;
  const int L = s.glen[r.group];
  r.pg0 = bt[2 * j];
  r.pg1 = (2 * j + 1 < p.max_pages) ? bt[2 * j + 1] : 0;
  r.two = (2 * j + 1) * kPage < L;
  return r;
}

// sum_h ReLU(v[h]) * w[h] over the 64 heads of one token is formed in the
// per-row scorer's order: eight running sums, a_c over h = 4i + c and b_c
// over h = 32 + 4i + c (i = 0..7), then ((a0+b0)+(a1+b1)) + ((a2+b2)+(a3+b3)).
// Pairs of sums run as packed f32x2 FMAs / adds; each lane of a packed
// operation is the scalar one.
__device__ __forceinline__ float2 relu2(uint32_t x, uint32_t y) {
  return make_float2(fmaxf(__uint_as_float(x), 0.f), fmaxf(__uint_as_float(y), 0.f));
}

// Adds 32 heads of one token into a pair of packed running sums (x01 over
// heads 4i, 4i+1; x23 over 4i+2, 4i+3).
__device__ __forceinline__ void head_part(const uint32_t (&v)[32], const float4* w4, float2& x01, float2& x23) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 w = w4[i];
    x01 = __ffma2_rn(relu2(v[4 * i + 0], v[4 * i + 1]), make_float2(w.x, w.y), x01);
    x23 = __ffma2_rn(relu2(v[4 * i + 2], v[4 * i + 3]), make_float2(w.z, w.w), x23);
  }
}

__device__ __forceinline__ float head_total(float2 a01, float2 a23, float2 b01, float2 b23) {
  const float2 s01 = __fadd2_rn(a01, b01), s23 = __fadd2_rn(a23, b23);
  return (s01.x + s01.y) + (s23.x + s23.y);
}

template <int R>
__global__ void __launch_bounds__(MqTraits<R>::kThreads, 1)
    score_mq_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                    const __grid_constant__ CUtensorMap tmap_s, const MqParams p) {
  using Tr = MqTraits<R>;
  constexpr int kN = Tr::kN, kAccs = Tr::kAccs, kEpiWarps = Tr::kEpiWarps, kMqStages = Tr::kStages;
  constexpr bool kSplitLoad = Tr::kThreads > 448;  // fewer than 128 registers a thread
  extern __shared__ uint8_t smem_raw[];
  MqSmem<R>& s = *reinterpret_cast<MqSmem<R>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  // Launched as a programmatic dependent: the barriers and the tensor-map
  // prefetch (shared memory and kernel parameters only) overlap the previous
  // kernel's tail; global memory is touched only after the wait.  (TMEM is
  // allocated after it: a predecessor still running on this SM may need it.)
  if (tid == 0) {
    for (int i = 0; i < kMqStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < kMqScaleSlots; ++i) {
      mbar_init(&s.sfull[i], 1);
      mbar_init(&s.sempty[i], kEpiWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.qfull[i], 1);
      mbar_init(&s.qempty[i], 1);
      mbar_init(&s.wfull[i], 1);
      mbar_init(&s.wempty[i], kEpiWarps);
    }
    for (int i = 0; i < kAccs; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], kEpiWarps);
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
  build_group_table(s, p);
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kMqTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  const int groups = p.rows / R;
  const int* gs = s.gstart;
  const int T = gs[groups];
  const int t0 = static_cast<int>((static_cast<long long>(T) * blockIdx.x) / gridDim.x);
  const int t1 = static_cast<int>((static_cast<long long>(T) * (blockIdx.x + 1)) / gridDim.x);

  if (t0 < t1) {
    if (warp == 0) {
      // ------------------------------------------------------------ producer
      const uint64_t pol_k = l2_policy_evict_first();
      const uint64_t pol_q = l2_policy_evict_last();
      int stage = 0, sslot = 0, qs = 1, cur_group = -1;
      uint32_t phase = 0, sphase = 0;
      uint32_t qe_par[2] = {0u, 0u};
      int q_uses[2] = {0, 0};
      int k_fills = 0, s_fills = 0;
      bool ok = true;
      GroupTile nxt = {0, 0, 0, 0};
      if (t0 + lane < t1) nxt = resolve_group_tile(s, p, t0 + lane);
      for (int tb = t0; tb < t1 && ok; tb += 32) {
        const GroupTile cur = nxt;
        // Resolve the next batch now; its loads overlap this batch's issue.
        if (tb + 32 + lane < t1) nxt = resolve_group_tile(s, p, tb + 32 + lane);
        if (tb + lane < t1 &&
            (static_cast<unsigned>(cur.pg0) >= static_cast<unsigned>(p.num_pages) ||
             (cur.two && static_cast<unsigned>(cur.pg1) >= static_cast<unsigned>(p.num_pages))))
          report(p.status, DSAI_STATUS_BAD_PAGE);  // TMA zero-fills out-of-range pages
        const int n = min(32, t1 - tb);
        for (int i = 0; i < n; ++i) {
          const int g = __shfl_sync(0xffffffffu, cur.group, i);
          const int a = __shfl_sync(0xffffffffu, cur.pg0, i);
          const int b = __shfl_sync(0xffffffffu, cur.pg1, i);
          const int tw = __shfl_sync(0xffffffffu, cur.two, i);
          int good = 1;
          if (lane == 0) {
            if (g != cur_group) {
              cur_group = g;
              qs ^= 1;
              // The slot's queries are free once the MMAs of its last group
              // completed, its weights once every epilogue warp left it.
              if (!mbar_wait(&s.qempty[qs], qe_par[qs] ^ 1u, &s.abort, kWaitTimeoutNs) ||
                  !mbar_wait(&s.wempty[qs], qe_par[qs] ^ 1u, &s.abort, kWaitTimeoutNs)) {
                good = 0;
              } else {
                qe_par[qs] ^= 1u;
                ++q_uses[qs];
                mbar_arrive_expect_tx(&s.qfull[qs], R * kQBytes);
#pragma unroll
                for (int r = 0; r < R; ++r)
                  tma_load_2d(s.q[qs] + r * kQBytes, &tmap_q, &s.qfull[qs], 0,
                              (p.row_base + g * R + r) * kHeads, pol_q);
                mbar_arrive_expect_tx(&s.wfull[qs], R * kHeads * 4);
                bulk_load(s.w[qs], p.weights + static_cast<size_t>(g) * R * kHeads, R * kHeads * 4,
                          &s.wfull[qs], pol_q);
              }
            }
            if (good && !mbar_wait(&s.empty[stage], phase ^ 1u, &s.abort, kWaitTimeoutNs)) good = 0;
            if (good && !mbar_wait(&s.sempty[sslot], sphase ^ 1u, &s.abort, kWaitTimeoutNs)) good = 0;
            if (good) {
              mbar_arrive_expect_tx(&s.full[stage], tw ? 2 * kPageKBytes : kPageKBytes);
              mbar_arrive_expect_tx(&s.sfull[sslot], tw ? 2 * kMqScaleTx : kMqScaleTx);
              tma_load_3d(s.k[stage], &tmap_k, &s.full[stage], 0, 0, a, pol_k);
              tma_load_2d(s.scale[sslot], &tmap_s, &s.sfull[sslot], 0, a, pol_k);
              if (tw) {
                tma_load_3d(s.k[stage] + kPageKBytes, &tmap_k, &s.full[stage], 0, 0, b, pol_k);
                tma_load_2d(s.scale[sslot] + kPage, &tmap_s, &s.sfull[sslot], 0, b, pol_k);
              }
              ++k_fills;
              ++s_fills;
              if (++stage == kMqStages) { stage = 0; phase ^= 1u; }
              if (++sslot == kMqScaleSlots) { sslot = 0; sphase ^= 1u; }
            } else {
              mq_fail(s, p.status);
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) { ok = false; break; }
        }
      }
      // Never leave with a copy in flight: wait for the latest fill of every
      // slot (each earlier fill of a slot was consumed, hence complete).
      if (lane == 0) {
        for (int i = 0; i < kMqStages && i < k_fills; ++i) {
          const int last = k_fills - 1 - i;
          if (!mbar_wait(&s.full[last % kMqStages], (last / kMqStages) & 1, nullptr, kWaitTimeoutNs))
            report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
        }
        for (int i = 0; i < kMqScaleSlots && i < s_fills; ++i) {
          const int last = s_fills - 1 - i;
          if (!mbar_wait(&s.sfull[last % kMqScaleSlots], (last / kMqScaleSlots) & 1, nullptr, kWaitTimeoutNs))
            report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
        }
        for (int i = 0; i < 2; ++i) {
          if (q_uses[i] > 0 && !mbar_wait(&s.qfull[i], (q_uses[i] - 1) & 1, nullptr, kWaitTimeoutNs))
            report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
          if (q_uses[i] > 0 && !mbar_wait(&s.wfull[i], (q_uses[i] - 1) & 1, nullptr, kWaitTimeoutNs))
            report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issuer
      if (lane == 0) {
        constexpr uint32_t idesc = make_idesc_e4m3_f32(kTileTok, kN);
        int stage = 0, acc = 0, qs = 1, cur_group = -1;
        uint32_t phase = 0, aphase = 0;
        uint32_t qf_par[2] = {0u, 0u};
        Cursor c;
        c.init(gs, groups, t0);
        for (; c.t < t1; c.next(gs, t1)) {
          if (c.row != cur_group) {
            if (cur_group >= 0) umma_commit(&s.qempty[qs]);  // previous group's queries free when done
            cur_group = c.row;
            qs ^= 1;
            if (!mbar_wait(&s.qfull[qs], qf_par[qs], &s.abort, kWaitTimeoutNs)) { mq_fail(s, p.status); break; }
            qf_par[qs] ^= 1u;
          }
          if (!mbar_wait(&s.full[stage], phase, &s.abort, kWaitTimeoutNs)) { mq_fail(s, p.status); break; }
          if (!mbar_wait(&s.tempty[acc], aphase ^ 1u, &s.abort, kWaitTimeoutNs)) { mq_fail(s, p.status); break; }
          tc_fence_after();
          const uint64_t adesc = make_sw128_kmajor_desc(smem_u32(s.k[stage]));
          const uint64_t bdesc = make_sw128_kmajor_desc(smem_u32(s.q[qs]));
          const uint32_t d = s.tmem_base + static_cast<uint32_t>(acc * kN);
#pragma unroll
          for (int kk = 0; kk < kDim / 32; ++kk)  // K = 32 e4m3 (32 B) per MMA
            umma_f8(d, adesc + 2u * kk, bdesc + 2u * kk, idesc, kk > 0 ? 1u : 0u);
          umma_commit(&s.empty[stage]);  // K stage free once these MMAs are done
          umma_commit(&s.tfull[acc]);
          if (++stage == kMqStages) { stage = 0; phase ^= 1u; }
          if (++acc == kAccs) { acc = 0; aphase ^= 1u; }
        }
        // Every MMA issued by this thread has completed once this arrives.
        umma_commit(&s.drain);
        if (!mbar_wait(&s.drain, 0, nullptr, kWaitTimeoutNs)) report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
      }
      __syncwarp();
    } else {
      // ------------------------------------------------------------ epilogue
      const int quad = warp & 3;                   // TMEM lanes [32*quad, 32*quad+32)
      const int r = (warp - 2) >> 2;               // the group row of this warp
      const int tok = quad * 32 + lane;            // token of the tile owned by this thread
      int acc = 0, sslot = 0, ws = 1, cur_group = -1, L = 0;
      uint32_t aphase = 0, sphase = 0;
      uint32_t wf_par[2] = {0u, 0u};
      size_t b = 0;
      Cursor c;
      c.init(gs, groups, t0);
      for (; c.t < t1; c.next(gs, t1)) {
        if (c.row != cur_group) {
          if (cur_group >= 0) {  // leaving a group: its weight slot is free for this warp
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.wempty[ws]);
          }
          cur_group = c.row;
          ws ^= 1;
          b = static_cast<size_t>(cur_group) * R + r;
          L = row_len(p.seq_lens, static_cast<int>(b), p.max_pages, nullptr);
          // Waits are decided warp-wide: the warp runs warp-collective steps below.
          if (!__all_sync(0xffffffffu, mbar_wait(&s.wfull[ws], wf_par[ws], &s.abort, kWaitTimeoutNs))) {
            mq_fail(s, p.status);
            break;
          }
          wf_par[ws] ^= 1u;
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&s.tfull[acc], aphase, &s.abort, kWaitTimeoutNs))) {
          mq_fail(s, p.status);
          break;
        }
        tc_fence_after();
        const uint32_t taddr = s.tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                               static_cast<uint32_t>(acc * kN + r * kHeads);
        const float4* w4 = reinterpret_cast<const float4*>(s.w[ws][r]);
        float2 a01 = make_float2(0.f, 0.f), a23 = a01, b01 = a01, b23 = a01;
        if constexpr (kSplitLoad) {
          // 32 columns at a time (the register budget of 4R warps)
          uint32_t v[32];
          tmem_ld_32x32b_x32(taddr, v);
          tmem_wait_ld();
          head_part(v, w4, a01, a23);
          tmem_ld_32x32b_x32(taddr + 32u, v);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tempty[acc]);
          head_part(v, w4 + 8, b01, b23);
        } else {
          uint32_t v0[32], v1[32];
          tmem_ld_32x32b_x32(taddr, v0);
          tmem_ld_32x32b_x32(taddr + 32u, v1);
          tmem_wait_ld();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.tempty[acc]);
          head_part(v0, w4, a01, a23);
          head_part(v1, w4 + 8, b01, b23);
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&s.sfull[sslot], sphase, &s.abort, kWaitTimeoutNs))) {
          mq_fail(s, p.status);
          break;
        }
        const float sc = s.scale[sslot][tok];
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.sempty[sslot]);
        const float logit = head_total(a01, a23, b01, b23) * sc;
        const int t_abs = c.j * kTileTok + tok;
        const bool live = t_abs < L;
        if (live) p.logits[b * p.ld + t_abs] = logit;
        if (L > kTopK) {
          // One reduction per token: with 4R epilogue warps sharing the issue
          // slots, aggregating equal bins in the warp first (the per-row
          // scorer's match) costs more than the L2 reductions it saves.
          const uint32_t bin = ordered_key(logit) >> (32 - kHistBits);
          if (live) atomicAdd(p.hist + static_cast<size_t>(b) * kHistStride + bin, 1u);  // RED
        }
        if (++acc == kAccs) { acc = 0; aphase ^= 1u; }
        if (++sslot == kMqScaleSlots) { sslot = 0; sphase ^= 1u; }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(s.tmem_base, kMqTmemCols);
  }
}

template <int R>
cudaError_t launch_mq(const ScoreLaunch& lp, const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& ts,
                      cudaStream_t stream) {
  static bool attr_set[64] = {};  // the attribute is per function and device
  int dev = 0;
  cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return e0;
  constexpr int kSmem = mq_smem_bytes<R>();
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(score_mq_kernel<R>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  MqParams p;
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(lp.grid);
  cfg.blockDim = dim3(MqTraits<R>::kThreads);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return launch_kernel(cfg, score_mq_kernel<R>, tq, tk, ts, p);
}

}  // namespace

cudaError_t launch_score_groups(const ScoreLaunch& lp, int rows_per_group, const CUtensorMap& tmap_q,
                                const CUtensorMap& tmap_k, const CUtensorMap& tmap_s, cudaStream_t stream) {
  if (rows_per_group < 2 || lp.rows % rows_per_group != 0 || lp.rows > kMaxRowsPerLaunch)
    return cudaErrorInvalidValue;
  switch (rows_per_group) {
    case 2: return launch_mq<2>(lp, tmap_q, tmap_k, tmap_s, stream);
    case 3: return launch_mq<3>(lp, tmap_q, tmap_k, tmap_s, stream);
    case 4: return launch_mq<4>(lp, tmap_q, tmap_k, tmap_s, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dsai
