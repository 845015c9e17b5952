// graph.h — launch recording and the CUDA-graph replay of a call's launches.
//
// Every kernel launch of the indexer's entry points goes through
// launch_kernel().  Normally that is cudaLaunchKernelEx.  While a
// LaunchRecorder is active on the calling thread, the launch is recorded
// instead: the kernel, its launch configuration and attributes, and a copy
// of its argument values.
//
// replay_recorded() turns a recorded call into one cudaGraphLaunch on the
// caller's stream.  Executable graphs are cached per (device, stream, launch
// plan): the kernels in order with their grid, block, dynamic shared memory
// and attributes.  Pointers and other argument values are not part of the
// key.  A miss captures the launches once, on a private capture stream, into
// a graph and instantiates it.  A hit writes the new argument values into the
// cached graph's kernel nodes (cudaGraphExecKernelNodeSetParams) and launches
// it.  This is the replay cache of the reference's host entry point
// (solution/python/kernel.cu:1101-1199, :1389-1478), which re-captures every
// call and splices it in with cudaGraphExecUpdate; here nothing is captured
// after the first call of a plan.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

namespace dsai {

constexpr int kRecMaxKernels = 8;    // launches of one call (score chunks + selection)
constexpr int kRecMaxArgs = 8;
constexpr int kRecArgBytes = 1024;   // three 128-B tensor maps and a parameter struct fit
constexpr int kRecMaxAttrs = 2;

struct KernelRecord {
  alignas(64) unsigned char args[kRecArgBytes];
  size_t arg_off[kRecMaxArgs];
  int nargs;
  const void* func;
  dim3 grid;
  dim3 block;
  size_t smem;
  cudaLaunchAttribute attrs[kRecMaxAttrs];
  int nattrs;
};

struct LaunchRecorder {
  KernelRecord recs[kRecMaxKernels];
  int n = 0;
  bool overflow = false;   // more launches, arguments or attributes than a record holds
};

// The recorder active on this thread (nullptr: launches run directly).
LaunchRecorder*& active_recorder();

// Activates `r` for the lifetime of the guard (nested guards restore the
// previous recorder).
class RecordScope {
 public:
  explicit RecordScope(LaunchRecorder* r) : prev_(active_recorder()) { active_recorder() = r; }
  ~RecordScope() { active_recorder() = prev_; }
  RecordScope(const RecordScope&) = delete;
  RecordScope& operator=(const RecordScope&) = delete;

 private:
  LaunchRecorder* prev_;
};

namespace detail {

template <typename T>
inline bool put_arg(KernelRecord& rec, size_t& off, const T& v) {
  off = (off + alignof(T) - 1) & ~(alignof(T) - 1);
  if (rec.nargs >= kRecMaxArgs || off + sizeof(T) > sizeof(rec.args)) return false;
  std::memcpy(rec.args + off, &v, sizeof(T));
  rec.arg_off[rec.nargs++] = off;
  off += sizeof(T);
  return true;
}

template <typename... KArgs>
cudaError_t record_launch(LaunchRecorder& r, const cudaLaunchConfig_t& cfg, void (*k)(KArgs...),
                          const KArgs&... vals) {
  if (r.n >= kRecMaxKernels || cfg.numAttrs > kRecMaxAttrs) {
    r.overflow = true;
    return cudaErrorNotSupported;
  }
  KernelRecord& rec = r.recs[r.n];
  rec.nargs = 0;
  size_t off = 0;
  bool ok = true;
  ((ok = ok && put_arg(rec, off, vals)), ...);
  if (!ok) {
    r.overflow = true;
    return cudaErrorNotSupported;
  }
  rec.func = reinterpret_cast<const void*>(k);
  rec.grid = cfg.gridDim;
  rec.block = cfg.blockDim;
  rec.smem = cfg.dynamicSmemBytes;
  rec.nattrs = static_cast<int>(cfg.numAttrs);
  for (int i = 0; i < rec.nattrs; ++i) rec.attrs[i] = cfg.attrs[i];
  ++r.n;
  return cudaSuccess;
}

}  // namespace detail

// cudaLaunchKernelEx, or a record of it while a LaunchRecorder is active.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(const cudaLaunchConfig_t& cfg, void (*k)(KArgs...), Args&&... args) {
  if (LaunchRecorder* r = active_recorder()) return detail::record_launch<KArgs...>(*r, cfg, k, args...);
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...);
}

// Launches the recorded kernels on `stream` as one cached executable graph
// (see above).  Returns cudaErrorNotSupported, having launched nothing, when
// the plan cannot be cached (the cache is full, or the capture failed); the
// caller then launches directly.
cudaError_t replay_recorded(const LaunchRecorder& r, cudaStream_t stream);

// Number of executable graphs in the cache (all devices and streams).
int graph_cache_entries();

}  // namespace dsai
