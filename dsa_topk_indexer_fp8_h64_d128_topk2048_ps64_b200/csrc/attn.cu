// attn.cu — sparse MLA attention over the indexer's top-2048 slots: the
// operator that consumes topk_indices in a DSA decode step (the contest
// operator dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64; its published
// definition: flashinfer 0.6.11.post2, flashinfer/trace/templates/
// attention.py, `_dsa_paged_reference`).
//
// For query token t and head h (16 heads), over the valid entries i of
// sparse_indices[t] (flat slot ids page*64 + slot, -1 = padding):
//   s_i = (q_nope[t,h] . ckv[i] + q_pe[t,h] . kpe[i]) * sm_scale
//   out[t,h] = sum_i softmax(s)_i ckv[i]   (bf16),  lse[t,h] = log2 sum_i exp(s_i)
// A token without a valid entry gets out = 0 and lse = -inf.
//
// HBM-bound: per token 2048 x (1024 + 128) B of gathered cache rows against
// 16 x 2048 x (576 + 512) x 2 flops.  One CTA per (token, split of its 2048
// entries); a split walks its entries in tiles of 64 rows:
//   warps 0-3  gather: each tile's 64 ckv rows (1 KB) and kpe rows (128 B)
//              with 16-B cp.async into a 128-B-swizzled [9 k-blocks][64 rows]
//              buffer (two buffers); -1 and out-of-range slots zero-fill.
//   warps 8-13 MMA issuers (one thread each; 4 for the scores, 2 for V^T P): S^T = K Q^T (tcgen05 kind::f16 M128 N16 K16, bf16
//              -> f32 in TMEM; rows 64-127 of the M = 128 operand are not
//              used) as four independent accumulator chains over the 36
//              K-steps (a single chain waits ~100 cycles per MMA on its
//              accumulator), then O^T += V^T P with the same buffer read
//              MN-major (64 ckv dims x 8 rows per 128-B atom) as the A operand.
//   warps 4-7  online softmax in base 2 (warps 4-5 own the 64 rows), P in
//              bf16 to shared memory, and at the end out = O / l,
//              lse = m + log2 l (or the split's (m, l, O) for the combine
//              kernel).  The reference maximum m moves only when a tile's
//              maximum exceeds it by more than 8 (then O^T in TMEM is
//              rescaled): probabilities stay <= 2^8, exact after the final
//              division, and the rescale, which must wait for the previous
//              tile's V^T P, is rare after the first tile.
#include <cuda_bf16.h>

#include <cmath>
#include <cstdio>

#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace dsai {
namespace {

using namespace sm100;

constexpr int kAHeads = DSAI_ATTN_HEADS;   // 16
constexpr int kACkv = DSAI_ATTN_CKV_DIM;   // 512
constexpr int kAKpe = DSAI_ATTN_KPE_DIM;   // 64
constexpr int kATopK = DSAI_TOPK;          // 2048
constexpr int kATile = 64;                 // cache rows per tile
constexpr int kAKBlocks = (kACkv + kAKpe) / 64;         // 9 k-blocks of 64 dims (128 B)
constexpr int kABlockBytes = kATile * 128;               // 8 KB
constexpr int kABufBytes = kAKBlocks * kABlockBytes;     // 72 KB
constexpr int kAQBlockBytes = kAHeads * 128;             // 2 KB
constexpr int kAQBytes = kAKBlocks * kAQBlockBytes;      // 18 KB
constexpr int kAPBytes = kAHeads * kATile * 2;           // 2 KB
constexpr int kASIssuers = 4;   // threads issuing the score MMAs (one accumulator chain each)
constexpr int kAOIssuers = 2;   // threads issuing the V^T P MMAs (two 128-dim blocks each)
constexpr int kAWarpS = 8;      // first score-issuer warp; the V^T P issuers follow
constexpr int kAThreads = 32 * (kAWarpS + kASIssuers + kAOIssuers);  // warps 0-3 gather, 4-7 softmax/epilogue
constexpr int kASChains = 4;     // partial score accumulators per tile
constexpr int kATmemCols = 256;  // S: 2 slots x 4 chains x 16 columns, O^T: 4 x 16 columns from column 128
constexpr int kAOCol = 2 * kASChains * kAHeads;
constexpr int kAMaxSplits = kATopK / kATile;  // 32
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;  // the reference maximum lags the true one by at most this

struct AttnParams {
  const uint8_t* q_nope;  // [T, 16, 512] bf16
  const uint8_t* q_pe;    // [T, 16, 64] bf16
  const uint8_t* ckv;     // [slots, 512] bf16
  const uint8_t* kpe;     // [slots, 64] bf16
  const int32_t* idx;     // [T, 2048]
  __nv_bfloat16* out;     // [T, 16, 512]
  float* lse;             // [T, 16]
  float* part_o;          // [T, splits, 16, 512] when splits > 1
  float* part_ml;         // [T, splits, 16, 2]
  int* status;
  float scale_log2;       // sm_scale * log2(e)
  int num_slots;
  int splits;
};

struct AttnSmem {
  uint8_t buf[2][kABufBytes];   // 1024-B aligned; A of S^T = K Q^T, A (MN-major) of O^T += V^T P
  uint8_t q[kAQBytes];          // B of S^T = K Q^T (K-major, 16 rows); also the tail read by the
                                // M = 128 operand of buffer 1's last k-block
  uint8_t p[2][kAPBytes];       // B of O^T += V^T P (K-major, 16 rows x 64 entries)
  float tmax[2][kAHeads];
  float tsum[2][kAHeads];
  float m[kAHeads];             // running maximum (log2 units)
  float l[kAHeads];             // running sum
  uint64_t full[2];             // tile gathered (128 producer arrivals)
  uint64_t done[2];             // O^T += V^T P of the tile in this slot completed (buffer and P free)
  uint64_t sfull[2];            // S^T of the tile in this slot in TMEM
  uint64_t pfull[2];            // P of the tile in this slot written (and O rescaled)
  uint64_t qfull;
  uint64_t drain[kASIssuers + kAOIssuers];  // per MMA-issuing thread
  uint32_t tmem_base;
  int abort;
  int fail_a;                   // epilogue failures before / after the tile's first named barrier
  int fail_b;
};

static_assert(kASIssuers == kASChains, "one score issuer per accumulator chain");
static_assert(4 % kAOIssuers == 0, "the V^T P issuers split the four 128-dim blocks");

constexpr int kAttnSmemBytes = static_cast<int>(sizeof(AttnSmem)) + 1024;
static_assert(kAttnSmemBytes <= 232448, "the attention CTA must fit");
static_assert(kAKBlocks * kABlockBytes + kABlockBytes <= kABufBytes + kAQBytes,
              "the M = 128 reads of buffer 1 stay inside the CTA's shared memory");

__device__ __forceinline__ void attn_fail(AttnSmem& s, int* status) {
  report(status, DSAI_STATUS_WAIT_TIMEOUT);
  *reinterpret_cast<volatile int*>(&s.abort) = 1;
}

// Reduces 16 per-lane values (one per head) over the 32 lanes of a warp by
// halving: at each step a lane keeps half of its values, sends the other
// half to its partner and combines, so 16 shuffles replace 16 x 5.  On
// return lane L holds the result for head 8*b4 + 4*b3 + 2*b2 + b1 (b =
// the bits of L); lanes L and L^1 hold the same head.
template <bool kMax>
__device__ __forceinline__ float warp_reduce16(const float (&v)[kAHeads], int lane) {
  float a[8];
  {
    const bool hi = lane & 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float send = hi ? v[j] : v[j + 8];
      const float keep = hi ? v[j + 8] : v[j];
      const float got = __shfl_xor_sync(0xffffffffu, send, 16);
      a[j] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
  float b[4];
  {
    const bool hi = lane & 8;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float send = hi ? a[j] : a[j + 4];
      const float keep = hi ? a[j + 4] : a[j];
      const float got = __shfl_xor_sync(0xffffffffu, send, 8);
      b[j] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
  float c[2];
  {
    const bool hi = lane & 4;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float send = hi ? b[j] : b[j + 2];
      const float keep = hi ? b[j + 2] : b[j];
      const float got = __shfl_xor_sync(0xffffffffu, send, 4);
      c[j] = kMax ? fmaxf(keep, got) : keep + got;
    }
  }
  float d;
  {
    const bool hi = lane & 2;
    const float send = hi ? c[0] : c[1];
    const float keep = hi ? c[1] : c[0];
    const float got = __shfl_xor_sync(0xffffffffu, send, 2);
    d = kMax ? fmaxf(keep, got) : keep + got;
  }
  const float got = __shfl_xor_sync(0xffffffffu, d, 1);
  return kMax ? fmaxf(d, got) : d + got;
}

__device__ __forceinline__ int reduce16_head(int lane) {
  return ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
}

// Byte offset of 16-B chunk `c` (0-7) of row `r` in a 128-B-swizzled atom
// column: the chunk index is XORed with the row's position in its 8-row group.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kAThreads, 1) attn_kernel(const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  AttnSmem& s = *reinterpret_cast<AttnSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t = blockIdx.y, split = blockIdx.x;
  const int entries = kATopK / p.splits;
  const int tiles = entries / kATile;
  const int32_t* idx_row = p.idx + static_cast<size_t>(t) * kATopK + static_cast<size_t>(split) * entries;

  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.full[i], 128);
      mbar_init(&s.done[i], kAOIssuers);  // every V^T P issuer commits
      mbar_init(&s.sfull[i], kASIssuers);  // every score issuer commits
      mbar_init(&s.pfull[i], 1);
    }
    mbar_init(&s.qfull, 128);
    for (int i = 0; i < kASIssuers + kAOIssuers; ++i) mbar_init(&s.drain[i], 1);
    for (int h = 0; h < kAHeads; ++h) {
      s.m[h] = -INFINITY;
      s.l[h] = 0.f;
    }
    s.abort = 0;
    s.fail_a = 0;
    s.fail_b = 0;
    fence_mbar_init();
  }
  if (warp == 8) {
    tmem_alloc(&s.tmem_base, kATmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = s.tmem_base;

  if (warp < 4) {
    // ------------------------------------------------------------ gather
    // Q: 16 heads x 72 chunks of 16 B (64 of q_nope, 8 of q_pe).
    for (int c = tid; c < kAHeads * 72; c += 128) {
      const int h = c / 72, cc = c % 72;
      const uint8_t* src = cc < 64 ? p.q_nope + (static_cast<size_t>(t) * kAHeads + h) * (kACkv * 2) + cc * 16
                                   : p.q_pe + (static_cast<size_t>(t) * kAHeads + h) * (kAKpe * 2) + (cc - 64) * 16;
      cp_async_16(s.q + (cc >> 3) * kAQBlockBytes + swz(h, cc & 7), src, 16);
    }
    cp_async_wait_all();
    fence_proxy_async_smem();
    mbar_arrive(&s.qfull);
    const int r0 = warp * 16;  // this warp's 16 rows of each tile
    int32_t next_id = lane < 16 && tiles > 0 ? idx_row[r0 + lane] : -1;  // one tile ahead
    for (int i = 0; i < tiles; ++i) {
      const int b = i & 1;
      const int32_t my_id = next_id;
      if (lane < 16 && i + 1 < tiles) next_id = idx_row[(i + 1) * kATile + r0 + lane];
      // The buffer is free once O^T += V^T P of the tile two back completed.
      if (!__all_sync(0xffffffffu, mbar_wait(&s.done[b], ((i >> 1) & 1) ^ 1u, &s.abort, kWaitTimeoutNs))) {
        if (lane == 0) attn_fail(s, p.status);
        break;
      }
      const bool my_ok = lane < 16 && my_id >= 0 && my_id < p.num_slots;
      if (lane < 16 && my_id != -1 && !my_ok) report(p.status, DSAI_STATUS_BAD_INDEX);
      uint8_t* bb = s.buf[b];
#pragma unroll 4
      for (int j = 0; j < 16; ++j) {
        const int id = __shfl_sync(0xffffffffu, my_id, j);
        const bool ok = __shfl_sync(0xffffffffu, my_ok ? 1 : 0, j) != 0;
        const int r = r0 + j;
        // invalid slots read nothing (src-size 0 zero-fills) from a valid address
        const uint8_t* crow = ok ? p.ckv + static_cast<size_t>(id) * (kACkv * 2) : p.ckv;
        const uint8_t* krow = ok ? p.kpe + static_cast<size_t>(id) * (kAKpe * 2) : p.kpe;
        const uint32_t nb = ok ? 16u : 0u;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int c = lane + 32 * hh;  // chunk 0-63 of the ckv row
          cp_async_16(bb + (c >> 3) * kABlockBytes + swz(r, c & 7), crow + c * 16, nb);
        }
        if (lane < 8) cp_async_16(bb + 8 * kABlockBytes + swz(r, lane), krow + lane * 16, nb);
      }
      cp_async_wait_all();
      fence_proxy_async_smem();
      mbar_arrive(&s.full[b]);
    }
  } else if (warp >= kAWarpS && warp < kAWarpS + kASIssuers) {
    // ------------------------------------------------------------ score MMA issuers
    // One thread per accumulator chain: the issue of a tcgen05.mma with
    // N = 16 costs its thread ~40 ns, so the 36 K-steps are spread.
    const int chain = warp - kAWarpS;
    if (lane == 0) {
      constexpr uint32_t idesc_s = make_idesc_bf16_f32(128, kAHeads, false);
      bool ok = mbar_wait(&s.qfull, 0, &s.abort, kWaitTimeoutNs);
      // The TMEM slot of tile i's scores was last read by the softmax of
      // tile i - 2, which finished before that tile's V^T P, which freed the
      // buffer this tile's rows came into.
      for (int i = 0; i < tiles && ok; ++i) {
        const int b = i & 1;
        if (!mbar_wait(&s.full[b], (i >> 1) & 1, &s.abort, kWaitTimeoutNs)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d = tbase + static_cast<uint32_t>(kASChains * kAHeads * (i & 1));
        const uint64_t a0 = make_sw128_kmajor_desc(smem_u32(s.buf[b]));
        const uint64_t q0 = make_sw128_kmajor_desc(smem_u32(s.q));
        // K-step n (16 dims) goes to chain n % 4; descriptor start addresses
        // advance in 16-B units
#pragma unroll 3
        for (int kb = 0; kb < kAKBlocks; ++kb) {  // this chain's K-steps n = 4 kb + chain
          const int n = kASChains * kb + chain, k16 = chain;
          const uint64_t a = a0 + static_cast<uint64_t>((kb * kABlockBytes + k16 * 32) >> 4);
          const uint64_t q = q0 + static_cast<uint64_t>((kb * kAQBlockBytes + k16 * 32) >> 4);
          umma_bf16(d + static_cast<uint32_t>(kAHeads * (n % kASChains)), a, q, idesc_s, n >= kASChains ? 1u : 0u);
        }
        umma_commit(&s.sfull[i & 1]);
      }
      if (!ok) attn_fail(s, p.status);
      // Every MMA issued by this thread has completed once this arrives.
      umma_commit(&s.drain[chain]);
      if (!mbar_wait(&s.drain[chain], 0, nullptr, kWaitTimeoutNs)) report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else if (warp >= kAWarpS + kASIssuers) {
    // ------------------------------------------------------------ V^T P MMA issuers
    // Threads of their own, so that a tile's V^T P (which frees the tile's
    // buffer) never waits behind the next tile's score MMAs.
    const int oi = warp - kAWarpS - kASIssuers;
    if (lane == 0) {
      constexpr uint32_t idesc_o = make_idesc_bf16_f32(128, kAHeads, true);
      bool ok = true;
      for (int i = 0; i < tiles; ++i) {
        if (!mbar_wait(&s.pfull[i & 1], (i >> 1) & 1, &s.abort, kWaitTimeoutNs)) { ok = false; break; }
        tc_fence_after();
        const int b = i & 1;
        const uint64_t v0 = make_sw128_mnmajor_desc(smem_u32(s.buf[b]), kABlockBytes);
        const uint64_t p0 = make_sw128_kmajor_desc(smem_u32(s.p[b]));
#pragma unroll
        for (int j = 0; j < kATile / 16; ++j) {  // 16 entries per MMA; this thread's M blocks interleave
#pragma unroll
          for (int mb = oi * (4 / kAOIssuers); mb < (oi + 1) * (4 / kAOIssuers); ++mb) {  // 128 dims each
            const uint64_t a = v0 + static_cast<uint64_t>(((2 * mb) * kABlockBytes + j * 2048) >> 4);
            const uint64_t pd = p0 + static_cast<uint64_t>((j * 32) >> 4);
            umma_bf16(tbase + static_cast<uint32_t>(kAOCol + 16 * mb), a, pd, idesc_o, (i > 0 || j > 0) ? 1u : 0u);
          }
        }
        umma_commit(&s.done[b]);
      }
      if (!ok) attn_fail(s, p.status);
      umma_commit(&s.drain[kASIssuers + oi]);
      if (!mbar_wait(&s.drain[kASIssuers + oi], 0, nullptr, kWaitTimeoutNs)) report(p.status, DSAI_STATUS_WAIT_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax / epilogue (warps 4-7)
    const int ep = tid - 128;
    const int quad = warp & 3;         // TMEM lanes [32 quad, 32 quad + 32)
    const bool sm = warp < 6;          // warps 4-5: the tile's 64 rows
    const int row = (warp - 4) * 32 + lane;
    volatile int* fail_a = &s.fail_a;
    volatile int* fail_b = &s.fail_b;
    bool finished = true;
    int32_t next_id = sm && tiles > 0 ? idx_row[row] : -1;  // one tile ahead
    for (int i = 0; i < tiles; ++i) {
      const int k = i & 1;
      // A: scaled scores of the tile's rows and the tile maximum per head
      float x[kAHeads];
      if (sm) {
        const int32_t id = next_id;
        if (i + 1 < tiles) next_id = idx_row[(i + 1) * kATile + row];
        const bool ok = id >= 0 && id < p.num_slots;
        const bool got = __all_sync(0xffffffffu, mbar_wait(&s.sfull[k], (i >> 1) & 1, &s.abort, kWaitTimeoutNs));
        if (got) {
          tc_fence_after();
          // the four partial sums, two chains at a time: (c0 + c1) + (c2 + c3)
          const uint32_t ta = tbase + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(kASChains * kAHeads * k);
          float half[kAHeads];
#pragma unroll
          for (int c = 0; c < kASChains; c += 2) {
            uint32_t r0[16], r1[16];
            tmem_ld_32x32b_x16(ta + static_cast<uint32_t>(kAHeads * c), r0);
            tmem_ld_32x32b_x16(ta + static_cast<uint32_t>(kAHeads * (c + 1)), r1);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < kAHeads; ++h) {
              const float sp = __uint_as_float(r0[h]) + __uint_as_float(r1[h]);
              if (c == 0) half[h] = sp; else x[h] = ok ? (half[h] + sp) * p.scale_log2 : -INFINITY;
            }
          }
        } else {
          if (lane == 0) { *fail_a = 1; attn_fail(s, p.status); }
#pragma unroll
          for (int h = 0; h < kAHeads; ++h) x[h] = -INFINITY;
        }
        const float mx = warp_reduce16<true>(x, lane);
        if ((lane & 1) == 0) s.tmax[warp - 4][reduce16_head(lane)] = mx;
      }
      named_bar_sync(1, 128);
      if (*fail_a) { finished = false; break; }
      // B: new running maximum, P, rescale of O^T
      float mnew[kAHeads], alpha[kAHeads];
      bool grow = false;  // O^T holds earlier tiles that need rescaling
#pragma unroll
      for (int h = 0; h < kAHeads; ++h) {
        const float mo = s.m[h];
        const float mt = fmaxf(s.tmax[0][h], s.tmax[1][h]);
        const float mn = (mo == -INFINITY || mt > mo + kRescaleLog2) ? fmaxf(mo, mt) : mo;
        mnew[h] = mn;
        // before the first valid entry O and l are zero: nothing to rescale
        alpha[h] = (mo == -INFINITY || mn == mo) ? 1.f : exp2f(mo - mn);
        grow |= mo != -INFINITY && mn != mo;
      }
      if (sm) {
        // this P slot was last read by O^T += V^T P of tile i - 2
        const bool freed = i < 2 || __all_sync(0xffffffffu, mbar_wait(&s.done[k], ((i >> 1) & 1) ^ 1u, &s.abort, kWaitTimeoutNs));
        if (!freed && lane == 0) { *fail_b = 1; attn_fail(s, p.status); }
        uint8_t* pk = s.p[k];
        float pr[kAHeads];
#pragma unroll
        for (int h = 0; h < kAHeads; ++h) {
          const float pv = x[h] == -INFINITY ? 0.f : ex2_approx(x[h] - mnew[h]);
          const __nv_bfloat16 pb = __float2bfloat16_rn(pv);
          if (freed)
            *reinterpret_cast<__nv_bfloat16*>(pk + swz(h, row >> 3) + (row & 7) * 2) = pb;
          pr[h] = pv;  // l in fp32 (as the reference's softmax); only the MMA operand is bf16
        }
        const float sum = warp_reduce16<false>(pr, lane);
        if ((lane & 1) == 0) s.tsum[warp - 4][reduce16_head(lane)] = sum;
        fence_proxy_async_smem();
      }
      if (i > 0 && grow) {
        // O^T holds tiles 0..i-1 once their last MMA (tile i-1) completed
        const bool got = __all_sync(0xffffffffu, mbar_wait(&s.done[(i - 1) & 1], ((i - 1) >> 1) & 1, &s.abort, kWaitTimeoutNs));
        if (got) {
          tc_fence_after();
#pragma unroll
          for (int mb = 0; mb < 4; ++mb) {
            uint32_t r[16];
            const uint32_t ta = tbase + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(kAOCol + 16 * mb);
            tmem_ld_32x32b_x16(ta, r);
            tmem_wait_ld();
#pragma unroll
            for (int h = 0; h < kAHeads; ++h) r[h] = __float_as_uint(__uint_as_float(r[h]) * alpha[h]);
            tmem_st_32x32b_x16(ta, r);
          }
          tmem_wait_st();
        } else if (lane == 0) {
          *fail_b = 1;
          attn_fail(s, p.status);
        }
      }
      tc_fence_before();
      named_bar_sync(1, 128);
      if (*fail_b) { finished = false; break; }
      if (warp == 4) {  // one head per lane, then hand the tile to the MMA issuer
        if (lane < kAHeads) {
          float al = 1.f, mn = 0.f;
#pragma unroll
          for (int h = 0; h < kAHeads; ++h)
            if (h == lane) { al = alpha[h]; mn = mnew[h]; }
          s.l[lane] = s.l[lane] * al + s.tsum[0][lane] + s.tsum[1][lane];
          s.m[lane] = mn;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.pfull[k]);
      }
    }
    if (finished && tiles > 0) {
      const bool got = __all_sync(0xffffffffu, mbar_wait(&s.done[(tiles - 1) & 1], ((tiles - 1) >> 1) & 1, &s.abort, kWaitTimeoutNs));
      named_bar_sync(1, 128);  // s.m / s.l of the last tile are final
      if (got) {
        tc_fence_after();
        float lh[kAHeads];
#pragma unroll
        for (int h = 0; h < kAHeads; ++h) lh[h] = s.l[h];
#pragma unroll
        for (int mb = 0; mb < 4; ++mb) {
          uint32_t r[16];
          tmem_ld_32x32b_x16(tbase + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(kAOCol + 16 * mb), r);
          tmem_wait_ld();
          const int d = 128 * mb + 32 * quad + lane;
          if (p.splits == 1) {
#pragma unroll
            for (int h = 0; h < kAHeads; ++h)
              p.out[(static_cast<size_t>(t) * kAHeads + h) * kACkv + d] =
                  __float2bfloat16_rn(lh[h] > 0.f ? __uint_as_float(r[h]) / lh[h] : 0.f);
          } else {
            float* po = p.part_o + (static_cast<size_t>(t) * p.splits + split) * kAHeads * kACkv;
#pragma unroll
            for (int h = 0; h < kAHeads; ++h) po[h * kACkv + d] = __uint_as_float(r[h]);
          }
        }
        if (ep < kAHeads) {
          const float mh = s.m[ep], lv = s.l[ep];
          if (p.splits == 1) {
            p.lse[static_cast<size_t>(t) * kAHeads + ep] = lv > 0.f ? mh + log2f(lv) : -INFINITY;
          } else {
            float* pm = p.part_ml + ((static_cast<size_t>(t) * p.splits + split) * kAHeads + ep) * 2;
            pm[0] = mh;
            pm[1] = lv;
          }
        }
      } else if (lane == 0) {
        attn_fail(s, p.status);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 8) {
    tc_fence_after();
    tmem_dealloc(tbase, kATmemCols);
  }
}

// Merges the splits of each (token, head), one CTA each:
// out = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
__global__ void __launch_bounds__(kACkv) attn_combine_kernel(const float* part_o, const float* part_ml, int splits,
                                                             __nv_bfloat16* out, float* lse) {
  const int h = blockIdx.x, t = blockIdx.y, d = threadIdx.x;
  {
    float mx = -INFINITY;
    for (int sp = 0; sp < splits; ++sp)
      mx = fmaxf(mx, part_ml[((static_cast<size_t>(t) * splits + sp) * kAHeads + h) * 2]);
    float num = 0.f, den = 0.f;
    for (int sp = 0; sp < splits; ++sp) {
      const size_t base = (static_cast<size_t>(t) * splits + sp) * kAHeads + h;
      const float ms = part_ml[base * 2], ls = part_ml[base * 2 + 1];
      const float w = ls > 0.f ? exp2f(ms - mx) : 0.f;
      num += w * part_o[base * kACkv + d];
      den += w * ls;
    }
    out[(static_cast<size_t>(t) * kAHeads + h) * kACkv + d] = __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
    if (d == 0) lse[static_cast<size_t>(t) * kAHeads + h] = den > 0.f ? mx + log2f(den) : -INFINITY;
  }
}

int attn_sms() {
  static int sm_count[64] = {};
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
    if (sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (sm_count[dev] > 0) sms = sm_count[dev];
  }
  return sms;
}

}  // namespace

int attn_splits(int num_tokens) {
  if (num_tokens <= 0) return 1;
  const int want = attn_sms() / num_tokens;  // CTAs of one wave per token
  int sp = 1;
  while (sp * 2 <= want && sp * 2 <= kAMaxSplits) sp *= 2;
  return sp;
}

size_t attn_workspace_bytes(int num_tokens) {
  const int sp = attn_splits(num_tokens);
  if (num_tokens <= 0) return kWsHeader;
  if (sp == 1) return kWsHeader;
  const size_t parts = static_cast<size_t>(num_tokens) * sp * kAHeads;
  return kWsHeader + parts * kACkv * sizeof(float) + parts * 2 * sizeof(float);
}

cudaError_t launch_attn(const AttnLaunch& a, cudaStream_t stream) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return e0;
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmemBytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int sp = attn_splits(a.num_tokens);
  AttnParams p;
  p.q_nope = static_cast<const uint8_t*>(a.q_nope);
  p.q_pe = static_cast<const uint8_t*>(a.q_pe);
  p.ckv = static_cast<const uint8_t*>(a.ckv);
  p.kpe = static_cast<const uint8_t*>(a.kpe);
  p.idx = a.idx;
  p.out = static_cast<__nv_bfloat16*>(a.out);
  p.lse = a.lse;
  uint8_t* ws = static_cast<uint8_t*>(a.workspace);
  const size_t parts = static_cast<size_t>(a.num_tokens) * sp * kAHeads;
  p.part_o = sp > 1 ? reinterpret_cast<float*>(ws + kWsHeader) : nullptr;
  p.part_ml = sp > 1 ? reinterpret_cast<float*>(ws + kWsHeader + parts * kACkv * sizeof(float)) : nullptr;
  p.status = reinterpret_cast<int*>(ws);
  p.scale_log2 = a.sm_scale * kLog2e;
  p.num_slots = a.num_slots;
  p.splits = sp;
  attn_kernel<<<dim3(sp, a.num_tokens), kAThreads, kAttnSmemBytes, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || sp == 1) return e;
  attn_combine_kernel<<<dim3(kAHeads, a.num_tokens), kACkv, 0, stream>>>(p.part_o, p.part_ml, sp, p.out, p.lse);
  return cudaGetLastError();
}

}  // namespace dsai

extern "C" DSAI_API size_t dsai_sparse_attn_workspace_size(int32_t num_tokens) {
  return num_tokens < 0 ? 0 : dsai::attn_workspace_bytes(num_tokens);
}

extern "C" DSAI_API int dsai_sparse_attn(const dsai_attn_args* a, void* workspace, size_t workspace_bytes,
                                         void* stream) {
  if (!a) return dsai::set_last_error(DSAI_E_INVALID, "args is NULL");
  if (a->num_tokens < 0 || a->num_pages < 0) return dsai::set_last_error(DSAI_E_INVALID, "negative size");
  if (a->num_tokens > 65535) return dsai::set_last_error(DSAI_E_INVALID, "num_tokens above 65535");
  if (a->num_tokens == 0) return DSAI_OK;
  if (!a->q_nope || !a->q_pe || !a->ckv_cache || !a->kpe_cache || !a->sparse_indices || !a->output || !a->lse)
    return dsai::set_last_error(DSAI_E_INVALID, "NULL pointer");
  const uintptr_t al = reinterpret_cast<uintptr_t>(a->q_nope) | reinterpret_cast<uintptr_t>(a->q_pe) |
                       reinterpret_cast<uintptr_t>(a->ckv_cache) | reinterpret_cast<uintptr_t>(a->kpe_cache);
  if (al % 16 != 0) return dsai::set_last_error(DSAI_E_INVALID, "q_nope, q_pe and the caches must be 16-B aligned");
  if (reinterpret_cast<uintptr_t>(a->sparse_indices) % 4 != 0 || reinterpret_cast<uintptr_t>(a->lse) % 4 != 0 ||
      reinterpret_cast<uintptr_t>(a->output) % 2 != 0)
    return dsai::set_last_error(DSAI_E_INVALID, "misaligned sparse_indices / output / lse");
  if (!std::isfinite(a->sm_scale)) return dsai::set_last_error(DSAI_E_INVALID, "sm_scale must be finite");
  if (static_cast<long long>(a->num_pages) * DSAI_PAGE_SIZE > 0x7fffffffll)
    return dsai::set_last_error(DSAI_E_INVALID, "num_pages too large");
  if (!workspace || reinterpret_cast<uintptr_t>(workspace) % 256 != 0)
    return dsai::set_last_error(DSAI_E_WORKSPACE, "workspace missing or not 256-B aligned");
  if (workspace_bytes < dsai::attn_workspace_bytes(a->num_tokens))
    return dsai::set_last_error(DSAI_E_WORKSPACE, "workspace smaller than dsai_sparse_attn_workspace_size()");
  dsai::AttnLaunch l;
  l.q_nope = a->q_nope;
  l.q_pe = a->q_pe;
  l.ckv = a->ckv_cache;
  l.kpe = a->kpe_cache;
  l.idx = a->sparse_indices;
  l.out = a->output;
  l.lse = a->lse;
  l.workspace = workspace;
  l.sm_scale = a->sm_scale;
  l.num_tokens = a->num_tokens;
  l.num_slots = a->num_pages * DSAI_PAGE_SIZE;
  const cudaError_t e = dsai::launch_attn(l, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "sparse attention launch: %s", cudaGetErrorString(e));
    return dsai::set_last_error(DSAI_E_CUDA, msg);
  }
  return DSAI_OK;
}
