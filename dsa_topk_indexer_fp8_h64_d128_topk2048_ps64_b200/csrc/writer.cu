// writer.cu — the index-K cache writer: per-token e4m3 quantisation of new
// keys and their scatter into the 8448-byte page layout the indexer reads.
//
// For each new token i with physical slot id s = slot_ids[i] (page*64 + slot,
// the id format of the indexer's output):
//   amax  = max_d |k[i,d]|, at least 1e-12
//   scale = amax / 448                                      (fp32)
//   q[d]  = e4m3(clamp(k[i,d] / scale, -448, 448))           (round to nearest even)
//   page bytes [slot*128, slot*128 + 128) <- q,  bytes 8192 + 4*slot <- scale
// which is the format of the index-K cache the reference consumes
// (solution/python/kernel.cu:29-40: 64 x 128 e4m3 then 64 fp32 scales per
// page).  Ids of -1 (padding) and ids outside [0, num_pages*64) are skipped.
//
// A half-warp per token: each lane loads 8 values (32 B of fp32 or 16 B of
// bf16), the half reduces the maximum with shuffles, and each lane stores 8
// bytes, so a token's 128-byte K row is one coalesced store; each half-warp
// keeps 2 tokens' loads in flight.  The kernel is
// HBM-bound: per token 512 (fp32) or 256 (bf16) bytes read, 4 bytes of id
// read and 132 bytes written.
#include <cuda_bf16.h>
#include <cuda_fp8.h>

#include <cstdio>

#include "common.cuh"
#include "launch.h"

namespace dsai {
namespace {

constexpr int kWriterThreads = 256;  // 8 warps per CTA
constexpr int kWriterCtasPerSm = 8;
constexpr int kTokPerHalf = 2;       // tokens a half-warp has in flight at once
constexpr int kTokPerWarp = 2 * kTokPerHalf;

// Quantises one token held by a half-warp (8 values per lane, lanes h16 =
// 0..15 of the half) and, when `live`, stores its 128-byte row and its
// scale.  Every lane of the warp runs it (its shuffles name the full warp).
__device__ __forceinline__ void store_token(const float (&v)[8], bool live, int32_t sid, int h16,
                                            uint8_t* k_cache) {
  float amax = 0.0f;
#pragma unroll
  for (int c = 0; c < 8; ++c) amax = fmaxf(amax, fabsf(v[c]));
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float scale = fmaxf(amax, 1e-12f) / 448.0f;
  // v / scale, correctly rounded, without a full division per element: with
  // y = RN(1/scale), q0 = RN(v*y) and the exact residual r = v - q0*scale
  // (one FMA), RN(q0 + r*y) is the correctly rounded quotient (Markstein,
  // IBM J. Res. Dev. 34(1), 1990, Theorem 1; scale is a normal positive
  // number and |v / scale| <= 448 here).  The correction step turns a -0
  // quotient into +0, so the sign of v (that of the quotient, scale > 0) is
  // put back.
  const float y = __frcp_rn(scale);
  uint32_t word[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float q[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float x = v[4 * h + c];
      const float q0 = x * y;
      const float r = fmaf(-q0, scale, x);
      q[c] = fminf(fmaxf(copysignf(fmaf(r, y, q0), x), -448.0f), 448.0f);
    }
    const __nv_fp8x2_storage_t lo = __nv_cvt_float2_to_fp8x2(make_float2(q[0], q[1]), __NV_SATFINITE, __NV_E4M3);
    const __nv_fp8x2_storage_t hi = __nv_cvt_float2_to_fp8x2(make_float2(q[2], q[3]), __NV_SATFINITE, __NV_E4M3);
    word[h] = static_cast<uint32_t>(lo) | (static_cast<uint32_t>(hi) << 16);
  }
  if (!live) return;
  const long long page = sid / kPage, slot = sid % kPage;
  uint8_t* pg = k_cache + page * kPageBytes;
  reinterpret_cast<uint2*>(pg + slot * kDim)[h16] = make_uint2(word[0], word[1]);
  if (h16 == 0) reinterpret_cast<float*>(pg + kScaleOff)[slot] = scale;
}

// Persistent grid; each half-warp takes kTokPerHalf tokens per step and
// issues all their loads (keys and ids) before it quantises any.
template <bool kBf16>
__global__ void __launch_bounds__(kWriterThreads)
    write_k_kernel(const void* __restrict__ k_new, const int32_t* __restrict__ slot_ids, int n,
                   uint8_t* __restrict__ k_cache, long long num_slots) {
  const int lane = threadIdx.x & 31, half = lane >> 4, h16 = lane & 15;
  const int warps = static_cast<int>(gridDim.x) * (kWriterThreads / 32);
  const int w = static_cast<int>(blockIdx.x) * (kWriterThreads / 32) + (threadIdx.x >> 5);
  for (int i0 = w * kTokPerWarp; i0 < n; i0 += warps * kTokPerWarp) {
    float v[kTokPerHalf][8];
    int32_t sid[kTokPerHalf];
#pragma unroll
    for (int u = 0; u < kTokPerHalf; ++u) {
      const int i = i0 + 2 * u + half;
      sid[u] = i < n ? slot_ids[i] : -1;
      if constexpr (kBf16) {
        uint4 raw = make_uint4(0u, 0u, 0u, 0u);
        if (i < n) raw = reinterpret_cast<const uint4*>(k_new)[static_cast<size_t>(i) * 16 + h16];
        const uint32_t wds[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wds[c]));
          v[u][2 * c] = f.x;
          v[u][2 * c + 1] = f.y;
        }
      } else {
        float4 x0 = make_float4(0.f, 0.f, 0.f, 0.f), x1 = x0;
        if (i < n) {
          const float4* src = reinterpret_cast<const float4*>(k_new) + static_cast<size_t>(i) * 32 + 2 * h16;
          x0 = src[0];
          x1 = src[1];
        }
        v[u][0] = x0.x; v[u][1] = x0.y; v[u][2] = x0.z; v[u][3] = x0.w;
        v[u][4] = x1.x; v[u][5] = x1.y; v[u][6] = x1.z; v[u][7] = x1.w;
      }
    }
#pragma unroll
    for (int u = 0; u < kTokPerHalf; ++u) {
      // padding (-1) and ids outside the pool are skipped
      const bool live = sid[u] >= 0 && static_cast<long long>(sid[u]) < num_slots;
      if (__any_sync(0xffffffffu, live)) store_token(v[u], live, sid[u], h16, k_cache);
    }
  }
}

}  // namespace

cudaError_t launch_write_k(const void* k_new, bool bf16, const int32_t* slot_ids, int n, uint8_t* k_cache,
                           int num_pages, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  static int sm_count[64] = {};  // per device, looked up once
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < 64) {
    if (sm_count[dev] == 0) cudaDeviceGetAttribute(&sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    if (sm_count[dev] > 0) sms = sm_count[dev];
  }
  const long long groups = (static_cast<long long>(n) + kTokPerWarp - 1) / kTokPerWarp;
  const long long need = (groups + kWriterThreads / 32 - 1) / (kWriterThreads / 32);
  const unsigned grid = static_cast<unsigned>(need < static_cast<long long>(sms) * kWriterCtasPerSm
                                                  ? need : static_cast<long long>(sms) * kWriterCtasPerSm);
  const long long num_slots = static_cast<long long>(num_pages) * kPage;
  if (bf16)
    write_k_kernel<true><<<grid, kWriterThreads, 0, stream>>>(k_new, slot_ids, n, k_cache, num_slots);
  else
    write_k_kernel<false><<<grid, kWriterThreads, 0, stream>>>(k_new, slot_ids, n, k_cache, num_slots);
  return cudaGetLastError();
}

}  // namespace dsai

extern "C" DSAI_API int dsai_write_k(const void* k_new, int32_t dtype, const int32_t* slot_ids, int32_t n_tokens,
                                     void* k_cache, int32_t num_pages, void* stream) {
  if (n_tokens < 0 || num_pages < 0) return dsai::set_last_error(DSAI_E_INVALID, "negative size");
  if (dtype != DSAI_DTYPE_F32 && dtype != DSAI_DTYPE_BF16)
    return dsai::set_last_error(DSAI_E_INVALID, "dtype must be DSAI_DTYPE_F32 or DSAI_DTYPE_BF16");
  if (n_tokens == 0) return DSAI_OK;
  if (!k_new || !slot_ids || !k_cache) return dsai::set_last_error(DSAI_E_INVALID, "NULL pointer");
  const uintptr_t need = dtype == DSAI_DTYPE_F32 ? 16 : 8;
  if (reinterpret_cast<uintptr_t>(k_new) % need != 0)
    return dsai::set_last_error(DSAI_E_INVALID, "k_new must be 16-B (fp32) / 8-B (bf16) aligned");
  if (reinterpret_cast<uintptr_t>(k_cache) % 16 != 0)
    return dsai::set_last_error(DSAI_E_INVALID, "k_cache must be 16-B aligned");
  const cudaError_t e = dsai::launch_write_k(k_new, dtype == DSAI_DTYPE_BF16, slot_ids, n_tokens,
                                             static_cast<uint8_t*>(k_cache), num_pages,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "index-K writer launch: %s", cudaGetErrorString(e));
    return dsai::set_last_error(DSAI_E_CUDA, msg);
  }
  return DSAI_OK;
}
