// api.cu — the C ABI (include/dsai.h): argument checks, TMA tensor maps,
// workspace layout and the launch sequence.
//
// Replaces the reference's host dispatcher dsa_topk_indexer_cuda
// (solution/python/kernel.cu:1208-1479).  Differences by design:
//   * explicit caller-owned workspace instead of a static per-device scratch
//     tensor (kernel.cu:1299-1323), so concurrent streams never share it;
//   * error codes + dsai_last_error() instead of exceptions;
//   * TMA tensor maps over the caller's buffers, encoded through the driver
//     entry point (no link-time dependency on libcuda).
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <climits>
#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "graph.h"
#include "launch.h"

namespace {

thread_local char g_err[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(DSAI_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceInfo {
  bool probed = false;
  bool sm100 = false;
  int sms = 0;
};
DeviceInfo g_dev[64];
std::mutex g_dev_mu;

int device_info(DeviceInfo* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(DSAI_E_UNSUPPORTED, "device index %d out of range", dev);
  std::lock_guard<std::mutex> g(g_dev_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.probed) {
    int major = 0, sms = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceGetAttribute");
    d.sm100 = (major == 10);
    d.sms = sms;
    d.probed = true;
  }
  *out = d;
  if (!d.sm100) return fail(DSAI_E_UNSUPPORTED, "device %d is not sm_100 (B200)", dev);
  return DSAI_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor maps of one call.  Encoding is a host-only computation (~1 us); the
// last few encodings are kept per thread, keyed by their arguments.
struct MapKey {
  const void* base;
  uint64_t extent;
  int kind;
  bool operator==(const MapKey& o) const {
    return base == o.base && extent == o.extent && kind == o.kind;
  }
};
struct MapEntry {
  MapKey key{nullptr, 0, -1};
  CUtensorMap map;
};
thread_local MapEntry g_maps[6];
thread_local int g_maps_next = 0;

enum MapKind { kMapQ = 0, kMapK = 1, kMapS = 2 };

int get_map(int kind, const void* base, uint64_t extent, CUtensorMap* out) {
  const MapKey key{base, extent, kind};
  for (auto& e : g_maps)
    if (e.key == key) {
      *out = e.map;
      return DSAI_OK;
    }
  auto enc = encode_fn();
  if (!enc) return fail(DSAI_E_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
  CUtensorMap m;
  CUresult r;
  if (kind == kMapQ) {  // q viewed as [rows*64, 128] bytes
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(dsai::kDim), extent};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(dsai::kDim)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(dsai::kDim), static_cast<cuuint32_t>(dsai::kHeads)};
    cuuint32_t es[2] = {1, 1};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (kind == kMapK) {  // K values viewed as [num_pages, 64, 128] bytes, page stride 8448
    cuuint64_t dims[3] = {static_cast<cuuint64_t>(dsai::kDim), static_cast<cuuint64_t>(dsai::kPage),
                          extent};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(dsai::kDim),
                             static_cast<cuuint64_t>(dsai::kPageBytes)};
    cuuint32_t box[3] = {static_cast<cuuint32_t>(dsai::kDim), static_cast<cuuint32_t>(dsai::kPage), 1};
    cuuint32_t es[3] = {1, 1, 1};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, es,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {  // scales viewed as [num_pages, 64] fp32 starting at byte 8192, page stride 8448
    const void* sbase = static_cast<const uint8_t*>(base) + dsai::kScaleOff;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(dsai::kPage), extent};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(dsai::kPageBytes)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(dsai::kPage), 1};
    cuuint32_t es[2] = {1, 1};
    r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(sbase), dims, strides, box,
            es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return fail(DSAI_E_CUDA, "cuTensorMapEncodeTiled(kind %d) failed: %d", kind, (int)r);
  MapEntry& e = g_maps[g_maps_next];
  g_maps_next = (g_maps_next + 1) % 6;
  e.key = key;
  e.map = m;
  *out = m;
  return DSAI_OK;
}

// Histogram rows known to be zero, per workspace.  Every call leaves the
// histograms of its `rows` rows zero, but its logits start right after them,
// so a later call with more rows finds the extra histogram rows dirty; those
// (and only those) are cleared before scoring.  dsai_workspace_init marks a
// whole workspace clean.
std::mutex g_ws_mu;
std::unordered_map<const void*, int32_t> g_ws_clean_rows;

int prepare_hist(void* ws, int32_t rows, cudaStream_t stream) {
  int32_t clean = 0;
  {
    std::lock_guard<std::mutex> g(g_ws_mu);
    auto it = g_ws_clean_rows.find(ws);
    if (it != g_ws_clean_rows.end()) clean = it->second;
    g_ws_clean_rows[ws] = rows;
  }
  if (rows > clean) {
    uint8_t* base = static_cast<uint8_t*>(ws) + dsai::kWsHeader +
                    static_cast<size_t>(clean) * dsai::kHistStride * sizeof(uint32_t);
    const size_t bytes = static_cast<size_t>(rows - clean) * dsai::kHistStride * sizeof(uint32_t);
    cudaError_t e = cudaMemsetAsync(base, 0, bytes, stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(histograms)");
  }
  return DSAI_OK;
}

// Workspaces whose logits region holds the fused launch's sentinel, with the
// geometry (rows, row stride) it was filled for.  The fused launch leaves the
// region so; any other launch that writes logits into it clears the entry.
struct SentinelGeom {
  int32_t rows;
  int32_t ld;
};
std::unordered_map<const void*, SentinelGeom> g_ws_sentinel;

void forget_sentinel(const void* ws) {
  std::lock_guard<std::mutex> g(g_ws_mu);
  g_ws_sentinel.erase(ws);
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Workspace layout: [header 256 B | per-row histogram blocks (4096 bins and
// 4 counters; 256-B rounded) | per-row pivot-bin lists of the split selection
// (kSplitCap keys, then kSplitCap values) | logits (256-B rounded)].
size_t hist_bytes(int32_t rows) {
  const size_t b = static_cast<size_t>(rows) * dsai::kHistStride * sizeof(uint32_t);
  return (b + 255) & ~static_cast<size_t>(255);
}

size_t cand_bytes(int32_t rows) {
  return static_cast<size_t>(rows) * dsai::kSplitCap * 2 * sizeof(uint32_t);
}

size_t logits_bytes(int32_t rows, int32_t max_pages) {
  const size_t b = static_cast<size_t>(rows) * static_cast<size_t>(max_pages) * dsai::kPage * sizeof(float);
  return (b + 255) & ~static_cast<size_t>(255);
}

uint32_t* ws_hist(void* ws) {
  return reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + dsai::kWsHeader);
}

uint32_t* ws_cand(void* ws, int32_t rows) {
  return reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(ws) + dsai::kWsHeader + hist_bytes(rows));
}

float* ws_logits(void* ws, int32_t rows) {
  return reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + dsai::kWsHeader + hist_bytes(rows) +
                                  cand_bytes(rows));
}

int check_args(const dsai_args* a, void* ws, size_t ws_bytes, bool need_ids) {
  if (!a) return fail(DSAI_E_INVALID, "args is NULL");
  if (a->rows < 0 || a->max_pages < 0 || a->num_pages < 0)
    return fail(DSAI_E_INVALID, "negative size (rows=%d max_pages=%d num_pages=%d)", a->rows,
                a->max_pages, a->num_pages);
  if (a->rows_per_seq < 0 || a->rows_per_seq > 4)
    return fail(DSAI_E_INVALID, "rows_per_seq must be 0 to 4 (got %d)", a->rows_per_seq);
  if (a->rows_per_seq > 1 && a->rows % a->rows_per_seq != 0)
    return fail(DSAI_E_INVALID, "rows (%d) must be a multiple of rows_per_seq (%d)", a->rows, a->rows_per_seq);
  if (a->rows == 0) return DSAI_OK;
  if (!a->seq_lens || !a->block_table) return fail(DSAI_E_INVALID, "seq_lens / block_table is NULL");
  if (need_ids && !a->topk_indices) return fail(DSAI_E_INVALID, "topk_indices is NULL");
  if (!aligned(a->topk_indices, 16)) return fail(DSAI_E_INVALID, "topk_indices must be 16-B aligned");
  if (!ws) return fail(DSAI_E_WORKSPACE, "workspace is NULL");
  if (!aligned(ws, 256)) return fail(DSAI_E_WORKSPACE, "workspace must be 256-B aligned");
  if (ws_bytes < dsai_workspace_size(a->rows, a->max_pages))
    return fail(DSAI_E_WORKSPACE, "workspace too small: %zu < %zu", ws_bytes,
                dsai_workspace_size(a->rows, a->max_pages));
  return DSAI_OK;
}

int check_scoring_args(const dsai_args* a) {
  if (!a->q || !a->k_cache || !a->weights) return fail(DSAI_E_INVALID, "q / k_cache / weights is NULL");
  if (a->num_pages < 1) return fail(DSAI_E_INVALID, "num_pages must be >= 1");
  if (!aligned(a->q, 16) || !aligned(a->k_cache, 16) || !aligned(a->weights, 16))
    return fail(DSAI_E_INVALID, "q, k_cache and weights must be 16-B aligned");
  if (a->logits_out && !aligned(a->logits_out, 16)) return fail(DSAI_E_INVALID, "logits_out must be 16-B aligned");
  if (static_cast<long long>(a->max_pages) * dsai::kPage > (1ll << 30))
    return fail(DSAI_E_INVALID, "max_pages too large");
  return DSAI_OK;
}

// The fused launch (fused.cu) serves batches of many independent rows that
// fit one launch: at least one row per four SMs (fewer rows are selected
// faster by several CTAs per row, select_split_kernel), rows scored one by
// one (rows_per_seq <= 1).
bool use_fused(const dsai_args* a, int sms) {
  const bool score_all = (a->flags & DSAI_FLAG_SCORE_ALL_ROWS) != 0;
  return dsai::fused_enabled() && a->rows <= dsai::kMaxRowsPerLaunch && a->rows_per_seq <= 1 &&
         static_cast<long long>(a->rows) * 4 >= sms && (!score_all || a->logits_out != nullptr);
}

// Scores all needed rows into `logits`, chunking by the per-launch row limit.
int run_scoring(const dsai_args* a, float* logits, uint32_t* hist, int* status, bool score_all, int sms,
                cudaStream_t stream) {
  CUtensorMap tq, tk, ts;
  int rc = get_map(kMapQ, a->q, static_cast<uint64_t>(a->rows) * dsai::kHeads, &tq);
  if (rc) return rc;
  rc = get_map(kMapK, a->k_cache, static_cast<uint64_t>(a->num_pages), &tk);
  if (rc) return rc;
  rc = get_map(kMapS, a->k_cache, static_cast<uint64_t>(a->num_pages), &ts);
  if (rc) return rc;
  const int ld = a->max_pages * dsai::kPage;
  const int group = a->rows_per_seq > 1 ? a->rows_per_seq : 1;
  const int chunk = (dsai::kMaxRowsPerLaunch / group) * group;  // launches never split a group
  for (int r0 = 0; r0 < a->rows; r0 += chunk) {
    const int n = a->rows - r0 < chunk ? a->rows - r0 : chunk;
    dsai::ScoreLaunch p;
    p.weights = a->weights + static_cast<size_t>(r0) * dsai::kHeads;
    p.seq_lens = a->seq_lens + r0;
    p.block_table = a->block_table + static_cast<size_t>(r0) * a->max_pages;
    p.logits = logits + static_cast<size_t>(r0) * ld;
    p.hist = hist + static_cast<size_t>(r0) * dsai::kHistStride;
    p.status = status;
    p.rows = n;
    p.max_pages = a->max_pages;
    p.num_pages = a->num_pages;
    p.ld = ld;
    p.row_base = r0;
    p.score_all = score_all ? 1 : 0;
    p.grid = sms;
    cudaError_t e = group > 1 ? dsai::launch_score_groups(p, group, tq, tk, ts, stream)
                              : dsai::launch_score(p, tq, tk, ts, stream);
    if (e != cudaSuccess) return cuda_fail(e, "score kernel launch");
  }
  return DSAI_OK;
}

// Whether `s` is capturing into a graph (a query that fails counts as
// capturing: the launches then go directly onto the stream).
bool stream_capturing(cudaStream_t s) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &st) != cudaSuccess) {
    cudaGetLastError();  // not the caller's error: clear it
    return true;
  }
  return st != cudaStreamCaptureStatusNone;
}

// Runs `plan` (a call's launches).  With `graph`, the launches are recorded
// and replayed from the cached executable graph of their plan; a plan that
// cannot be cached runs directly.
template <class F>
int run_launches(bool graph, cudaStream_t stream, F&& plan) {
  if (graph) {
    dsai::LaunchRecorder rec;
    int rc;
    {
      dsai::RecordScope scope(&rec);
      rc = plan();
    }
    if (rc == DSAI_OK) {
      const cudaError_t e = dsai::replay_recorded(rec, stream);
      if (e == cudaSuccess) return DSAI_OK;
      if (e != cudaErrorNotSupported) return cuda_fail(e, "CUDA graph replay");
    } else if (!rec.overflow) {
      return rc;
    }
  }
  return plan();
}

}  // namespace

namespace dsai {
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace dsai

extern "C" {

size_t dsai_workspace_size(int32_t rows, int32_t max_pages) {
  if (rows < 0 || max_pages < 0) return 0;
  return dsai::kWsHeader + hist_bytes(rows) + cand_bytes(rows) + logits_bytes(rows, max_pages);
}

int dsai_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace || workspace_bytes < dsai::kWsHeader) return fail(DSAI_E_WORKSPACE, "workspace too small");
  cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(workspace)");
  std::lock_guard<std::mutex> g(g_ws_mu);
  g_ws_clean_rows[workspace] = INT_MAX;
  g_ws_sentinel.erase(workspace);
  return DSAI_OK;
}

int dsai_run(const dsai_args* a, void* workspace, size_t workspace_bytes, void* stream_) {
  int rc = check_args(a, workspace, workspace_bytes, true);
  if (rc || a->rows == 0) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DeviceInfo dev;
  rc = device_info(&dev);
  if (rc) return rc;
  int* status = static_cast<int*>(workspace);
  const bool score_all = (a->flags & DSAI_FLAG_SCORE_ALL_ROWS) != 0;
  const bool all_short = static_cast<long long>(a->max_pages) * dsai::kPage <= dsai::kTopK;
  const bool graph = (a->flags & DSAI_FLAG_GRAPH) != 0 && !a->ev_after_score && !stream_capturing(stream);

  if (all_short && !score_all) {
    // No row can exceed the top-K: the answer does not depend on scores.
    if (a->ev_after_score) {
      cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(a->ev_after_score), stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    }
    return run_launches(graph, stream, [&]() -> int {
      cudaError_t e = dsai::launch_short_rows(a->seq_lens, a->block_table, a->rows, a->max_pages,
                                              a->topk_indices, stream);
      if (e != cudaSuccess) return cuda_fail(e, "short-rows kernel launch");
      return DSAI_OK;
    });
  }
  rc = check_scoring_args(a);
  if (rc) return rc;
  float* logits = a->logits_out ? a->logits_out : ws_logits(workspace, a->rows);
  uint32_t* hist = ws_hist(workspace);
  rc = prepare_hist(workspace, a->rows, stream);
  if (rc) return rc;
  if (use_fused(a, dev.sms)) {
    // Many independent rows: scoring and selection in one launch, each row
    // selected as soon as its scoring completes.
    CUtensorMap tq, tk, ts;
    rc = get_map(kMapQ, a->q, static_cast<uint64_t>(a->rows) * dsai::kHeads, &tq);
    if (rc) return rc;
    rc = get_map(kMapK, a->k_cache, static_cast<uint64_t>(a->num_pages), &tk);
    if (rc) return rc;
    rc = get_map(kMapS, a->k_cache, static_cast<uint64_t>(a->num_pages), &ts);
    if (rc) return rc;
    const int32_t ld = a->max_pages * dsai::kPage;
    const size_t lbytes = static_cast<size_t>(a->rows) * static_cast<size_t>(ld) * sizeof(float);
    const unsigned char sent = static_cast<unsigned char>(dsai::fused_logits_sentinel() & 0xFFu);
    bool fill = a->logits_out != nullptr;  // the caller's buffer: filled every call
    if (!fill) {
      std::lock_guard<std::mutex> g(g_ws_mu);
      auto it = g_ws_sentinel.find(workspace);
      fill = it == g_ws_sentinel.end() || it->second.rows != a->rows || it->second.ld != ld;
      g_ws_sentinel[workspace] = SentinelGeom{a->rows, ld};
    }
    if (fill) {
      cudaError_t e = cudaMemsetAsync(logits, sent, lbytes, stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(logits sentinel)");
    }
    dsai::FusedLaunch fp;
    fp.weights = a->weights;
    fp.seq_lens = a->seq_lens;
    fp.block_table = a->block_table;
    fp.logits = logits;
    fp.hist = hist;
    fp.keep_logits = a->logits_out != nullptr ? 1 : 0;
    fp.ws = status;
    fp.out_ids = a->topk_indices;
    fp.rows = a->rows;
    fp.max_pages = a->max_pages;
    fp.num_pages = a->num_pages;
    fp.ld = a->max_pages * dsai::kPage;
    fp.score_all = score_all ? 1 : 0;
    fp.sms = dev.sms;
    cudaError_t e = dsai::launch_fused(fp, tq, tk, ts, stream);
    if (e != cudaSuccess) return cuda_fail(e, "fused kernel launch");
    if (a->ev_after_score) {  // no boundary inside the fused launch: recorded after it
      e = cudaEventRecord(static_cast<cudaEvent_t>(a->ev_after_score), stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    }
    return DSAI_OK;
  }
  if (!a->logits_out) forget_sentinel(workspace);
  return run_launches(graph, stream, [&]() -> int {
    int rc2 = run_scoring(a, logits, hist, status, score_all, dev.sms, stream);
    if (rc2) return rc2;
    if (a->ev_after_score) {
      cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(a->ev_after_score), stream);
      if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
    }
    dsai::SelectLaunch sp;
    sp.logits = logits;
    sp.ld = a->max_pages * dsai::kPage;
    sp.hist = hist;
    sp.cand = ws_cand(workspace, a->rows);
    sp.seq_lens = a->seq_lens;
    sp.block_table = a->block_table;
    sp.rows = a->rows;
    sp.max_pages = a->max_pages;
    sp.status = status;
    sp.out_ids = a->topk_indices;
    sp.out_scores = nullptr;
    sp.out_tokens = nullptr;
    sp.token_offset = 0;
    sp.sms = dev.sms;
    cudaError_t e = dsai::launch_select(sp, stream);
    if (e != cudaSuccess) return cuda_fail(e, "select kernel launch");
    return DSAI_OK;
  });
}

int dsai_graph_cache_entries(void) { return dsai::graph_cache_entries(); }

int dsai_run_pairs(const dsai_args* a, int32_t token_offset, float* out_scores, int32_t* out_tokens,
                   void* workspace, size_t workspace_bytes, void* stream_) {
  int rc = check_args(a, workspace, workspace_bytes, false);
  if (rc || a->rows == 0) return rc;
  if (!out_scores || !out_tokens) return fail(DSAI_E_INVALID, "out_scores / out_tokens is NULL");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  DeviceInfo dev;
  rc = device_info(&dev);
  if (rc) return rc;
  rc = check_scoring_args(a);
  if (rc) return rc;
  int* status = static_cast<int*>(workspace);
  float* logits = a->logits_out ? a->logits_out : ws_logits(workspace, a->rows);
  uint32_t* hist = ws_hist(workspace);
  rc = prepare_hist(workspace, a->rows, stream);
  if (rc) return rc;
  if (!a->logits_out) forget_sentinel(workspace);
  rc = run_scoring(a, logits, hist, status, true, dev.sms, stream);
  if (rc) return rc;
  if (a->ev_after_score) {
    cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(a->ev_after_score), stream);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventRecord");
  }
  dsai::SelectLaunch sp;
  sp.logits = logits;
  sp.ld = a->max_pages * dsai::kPage;
  sp.hist = hist;
  sp.cand = ws_cand(workspace, a->rows);
  sp.seq_lens = a->seq_lens;
  sp.block_table = a->block_table;
  sp.rows = a->rows;
  sp.max_pages = a->max_pages;
  sp.status = status;
  sp.out_ids = nullptr;
  sp.out_scores = out_scores;
  sp.out_tokens = out_tokens;
  sp.token_offset = token_offset;
  sp.sms = dev.sms;
  cudaError_t e = dsai::launch_select(sp, stream);
  if (e != cudaSuccess) return cuda_fail(e, "select kernel launch");
  return DSAI_OK;
}

int dsai_merge_pairs(const float* scores, const int32_t* tokens, int32_t n_cand, const int32_t* bt_row,
                     int32_t max_pages, const int32_t* seq_len, int32_t* out, void* stream_) {
  if (n_cand < 0 || max_pages < 0) return fail(DSAI_E_INVALID, "negative size");
  if (!bt_row || !seq_len || !out || (n_cand > 0 && (!scores || !tokens)))
    return fail(DSAI_E_INVALID, "NULL pointer");
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  cudaError_t e = dsai::launch_merge(scores, tokens, n_cand, bt_row, max_pages, seq_len, out,
                                     static_cast<cudaStream_t>(stream_));
  if (e != cudaSuccess) return cuda_fail(e, "merge kernel launch");
  return DSAI_OK;
}

int dsai_read_status(void* workspace, void* stream_, int32_t* status_out) {
  if (!workspace || !status_out) return fail(DSAI_E_INVALID, "NULL pointer");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  int32_t v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, workspace, sizeof(v), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(workspace, 0, sizeof(int32_t), stream);
  if (e != cudaSuccess) return cuda_fail(e, "reading workspace status");
  *status_out = v;
  return DSAI_OK;
}

int dsai_selftest_wait_timeout(void* workspace, uint64_t timeout_ns, void* stream) {
  if (!workspace) return fail(DSAI_E_INVALID, "workspace is NULL");
  if (timeout_ns == 0 || timeout_ns > dsai::kWaitTimeoutNs) return fail(DSAI_E_INVALID, "timeout out of range");
  DeviceInfo dev;
  int rc = device_info(&dev);
  if (rc) return rc;
  cudaError_t e = dsai::launch_wait_selftest(static_cast<int*>(workspace), timeout_ns,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "self-test kernel launch");
  return DSAI_OK;
}

const char* dsai_last_error(void) { return g_err; }

const char* dsai_version(void) { return "dsai 0.1.0 (sm_100a)"; }

}  // extern "C"
