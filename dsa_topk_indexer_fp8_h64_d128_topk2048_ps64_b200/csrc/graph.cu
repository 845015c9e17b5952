// graph.cu — the per-(device, stream, launch plan) cache of executable CUDA
// graphs behind DSAI_FLAG_GRAPH (graph.h).
#include "graph.h"

#include <mutex>
#include <vector>

namespace dsai {

LaunchRecorder*& active_recorder() {
  thread_local LaunchRecorder* r = nullptr;
  return r;
}

namespace {

constexpr int kGraphCacheMax = 64;  // executable graphs kept (never evicted: one may be in flight)

// Attribute values compared field by field: the launchers leave the unused
// bytes of the value union uninitialised.
bool same_attr(const cudaLaunchAttribute& x, const cudaLaunchAttribute& y) {
  if (x.id != y.id) return false;
  switch (x.id) {
    case cudaLaunchAttributeProgrammaticStreamSerialization:
      return x.val.programmaticStreamSerializationAllowed == y.val.programmaticStreamSerializationAllowed;
    case cudaLaunchAttributeClusterDimension:
      return x.val.clusterDim.x == y.val.clusterDim.x && x.val.clusterDim.y == y.val.clusterDim.y &&
             x.val.clusterDim.z == y.val.clusterDim.z;
    default:
      return std::memcmp(&x.val, &y.val, sizeof(x.val)) == 0;
  }
}

bool same_dim(const dim3& a, const dim3& b) { return a.x == b.x && a.y == b.y && a.z == b.z; }

struct PlanKernel {
  const void* func;
  dim3 grid;
  dim3 block;
  size_t smem;
  int nattrs;
  cudaLaunchAttribute attrs[kRecMaxAttrs];
};

struct Plan {
  int device = -1;
  cudaStream_t stream = nullptr;
  int n = 0;
  PlanKernel k[kRecMaxKernels];

  bool matches(int dev, cudaStream_t s, const LaunchRecorder& r) const {
    if (device != dev || stream != s || n != r.n) return false;
    for (int i = 0; i < n; ++i) {
      const KernelRecord& rec = r.recs[i];
      const PlanKernel& pk = k[i];
      if (pk.func != rec.func || !same_dim(pk.grid, rec.grid) || !same_dim(pk.block, rec.block) ||
          pk.smem != rec.smem || pk.nattrs != rec.nattrs)
        return false;
      for (int j = 0; j < pk.nattrs; ++j)
        if (!same_attr(pk.attrs[j], rec.attrs[j])) return false;
    }
    return true;
  }
};

struct Entry {
  Plan plan;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  cudaGraphNode_t nodes[kRecMaxKernels] = {};
};

std::mutex g_mu;
std::vector<Entry*> g_entries;         // owned; released at process exit by the driver
cudaStream_t g_capture_stream[64] = {};

void arg_ptrs(const KernelRecord& rec, void** out) {
  for (int i = 0; i < rec.nargs; ++i)
    out[i] = const_cast<unsigned char*>(rec.args) + rec.arg_off[i];
}

cudaLaunchConfig_t config_of(const KernelRecord& rec, cudaStream_t stream, cudaLaunchAttribute* attrs) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = rec.grid;
  cfg.blockDim = rec.block;
  cfg.dynamicSmemBytes = rec.smem;
  cfg.stream = stream;
  for (int i = 0; i < rec.nattrs; ++i) attrs[i] = rec.attrs[i];
  cfg.attrs = attrs;
  cfg.numAttrs = static_cast<unsigned>(rec.nattrs);
  return cfg;
}

// Captures the recorded launches into a new graph on the device's private
// capture stream and instantiates it.  Returns the entry, or nullptr with
// `*err` set.
Entry* capture(int dev, cudaStream_t stream, const LaunchRecorder& r, cudaError_t* err) {
  if (!g_capture_stream[dev]) {
    cudaError_t e = cudaStreamCreateWithFlags(&g_capture_stream[dev], cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      g_capture_stream[dev] = nullptr;
      *err = e;
      return nullptr;
    }
  }
  cudaStream_t cs = g_capture_stream[dev];
  Entry* ent = new Entry();
  ent->plan.device = dev;
  ent->plan.stream = stream;
  ent->plan.n = r.n;
  cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
  cudaError_t first = e;
  if (e == cudaSuccess) {
    for (int i = 0; i < r.n && first == cudaSuccess; ++i) {
      const KernelRecord& rec = r.recs[i];
      void* argp[kRecMaxArgs];
      arg_ptrs(rec, argp);
      cudaLaunchAttribute attrs[kRecMaxAttrs];
      cudaLaunchConfig_t cfg = config_of(rec, cs, attrs);
      first = cudaLaunchKernelExC(&cfg, rec.func, argp);
      if (first != cudaSuccess) break;
      cudaStreamCaptureStatus st;
      const cudaGraphNode_t* deps = nullptr;
      const cudaGraphEdgeData* edges = nullptr;
      size_t nd = 0;
      first = cudaStreamGetCaptureInfo_v3(cs, &st, nullptr, nullptr, &deps, &edges, &nd);
      if (first == cudaSuccess && (st != cudaStreamCaptureStatusActive || nd != 1)) first = cudaErrorStreamCaptureInvalidated;
      if (first == cudaSuccess) ent->nodes[i] = deps[0];
      PlanKernel& pk = ent->plan.k[i];
      pk.func = rec.func;
      pk.grid = rec.grid;
      pk.block = rec.block;
      pk.smem = rec.smem;
      pk.nattrs = rec.nattrs;
      for (int j = 0; j < rec.nattrs; ++j) pk.attrs[j] = rec.attrs[j];
    }
    cudaGraph_t g = nullptr;
    e = cudaStreamEndCapture(cs, &g);  // always ends the capture, whatever failed inside it
    if (first == cudaSuccess) first = e;
    ent->graph = g;
  }
  if (first == cudaSuccess) first = cudaGraphInstantiateWithFlags(&ent->exec, ent->graph, 0);
  if (first != cudaSuccess) {
    if (ent->exec) cudaGraphExecDestroy(ent->exec);
    if (ent->graph) cudaGraphDestroy(ent->graph);
    delete ent;
    *err = first;
    return nullptr;
  }
  return ent;
}

}  // namespace

cudaError_t replay_recorded(const LaunchRecorder& r, cudaStream_t stream) {
  if (r.overflow || r.n <= 0) return cudaErrorNotSupported;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorNotSupported;
  // Held through the parameter update and the launch: the cached graph's
  // kernel nodes are shared by every thread calling with this stream.
  std::lock_guard<std::mutex> lock(g_mu);
  Entry* ent = nullptr;
  for (Entry* x : g_entries)
    if (x->plan.matches(dev, stream, r)) {
      ent = x;
      break;
    }
  if (!ent) {
    if (static_cast<int>(g_entries.size()) >= kGraphCacheMax) return cudaErrorNotSupported;
    ent = capture(dev, stream, r, &e);
    if (!ent) {
      // A plan that cannot be captured here (for instance another capture in
      // global mode on this device) is launched directly; a real launch
      // error shows up there.
      cudaGetLastError();
      return cudaErrorNotSupported;
    }
    g_entries.push_back(ent);
    return cudaGraphLaunch(ent->exec, stream);  // captured with this call's arguments
  }
  for (int i = 0; i < r.n; ++i) {
    const KernelRecord& rec = r.recs[i];
    void* argp[kRecMaxArgs];
    arg_ptrs(rec, argp);
    cudaKernelNodeParams kp = {};
    kp.func = const_cast<void*>(rec.func);
    kp.gridDim = rec.grid;
    kp.blockDim = rec.block;
    kp.sharedMemBytes = static_cast<unsigned>(rec.smem);
    kp.kernelParams = argp;
    kp.extra = nullptr;
    // Affects later launches only; a launch of this graph still running is not changed.
    e = cudaGraphExecKernelNodeSetParams(ent->exec, ent->nodes[i], &kp);
    if (e != cudaSuccess) return e;
  }
  return cudaGraphLaunch(ent->exec, stream);
}

int graph_cache_entries() {
  std::lock_guard<std::mutex> lock(g_mu);
  return static_cast<int>(g_entries.size());
}

}  // namespace dsai
