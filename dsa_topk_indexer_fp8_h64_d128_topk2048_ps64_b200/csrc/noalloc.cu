// noalloc.cu — the indexer for callers that cannot allocate device memory.
//
// dsai_run needs a caller-provided workspace.  Some callers have no way to
// provide one: a host that owns every device allocation through its own pool
// and forbids plugins to call cudaMalloc, a serving loop that bans allocation
// after warm-up (a cudaMalloc there can synchronise the device), or a binding
// from a language whose runtime has no device allocator.  For them this file
// keeps the workspace in a fixed device array that is part of the library
// image itself, so the call allocates nothing.
//
// Costs and limits, stated for the user:
//   * kNoAllocScratchBytes (16 MiB) of device memory is held on every GPU
//     that loads the library, until the process exits;
//   * a call whose dsai_workspace_size(rows, max_pages) exceeds it is
//     rejected with DSAI_E_WORKSPACE (B = 64 rows of up to 32K tokens fit);
//   * the first call on a device looks up the array's device address and
//     zeroes the array; make that first call before any stream capture;
//   * every call on a device shares the one array, which keeps the previous
//     call's contents: calls whose work can overlap on the GPU (other
//     streams, other host threads) race — serialise them.
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "launch.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t{16} << 20;

// The workspace of dsai_run_noalloc.  In host code this symbol is only a
// handle: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64];

// Looks up (once per device, with that device current) the scratch address
// and zeroes the scratch on `stream`.
int noalloc_setup(int dev, cudaStream_t stream, void** out) {
  std::lock_guard<std::mutex> g(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr)
      return dsai::set_last_error(DSAI_E_CUDA, "cudaGetSymbolAddress(static scratch) failed");
    const int rc = dsai_workspace_init(ptr, kNoAllocScratchBytes, stream);
    if (rc != DSAI_OK) return rc;
    g_noalloc_ptr[dev] = ptr;
  }
  *out = g_noalloc_ptr[dev];
  return DSAI_OK;
}

}  // namespace

extern "C" int dsai_run_noalloc(const dsai_args* args, void* stream_) {
  if (!args) return dsai::set_last_error(DSAI_E_INVALID, "args is NULL");
  if (args->rows < 0 || args->max_pages < 0 || args->num_pages < 0)
    return dsai::set_last_error(DSAI_E_INVALID, "negative size");
  const size_t need = dsai_workspace_size(args->rows, args->max_pages);
  if (need == 0 || need > kNoAllocScratchBytes) {
    char msg[160];
    snprintf(msg, sizeof(msg),
             "rows=%d, max_pages=%d need %zu bytes of workspace; the static scratch holds %zu",
             args->rows, args->max_pages, need, kNoAllocScratchBytes);
    return dsai::set_last_error(DSAI_E_WORKSPACE, msg);
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return dsai::set_last_error(DSAI_E_CUDA, "no current CUDA device");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  void* ws = nullptr;
  const int rc = noalloc_setup(dev, stream, &ws);
  if (rc != DSAI_OK) return rc;
  return dsai_run(args, ws, kNoAllocScratchBytes, stream_);
}

extern "C" int dsai_noalloc_read_status(void* stream, int32_t* status_out) {
  if (!status_out) return dsai::set_last_error(DSAI_E_INVALID, "status_out is NULL");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return dsai::set_last_error(DSAI_E_CUDA, "no current CUDA device");
  void* ws = nullptr;
  {
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    ws = g_noalloc_ptr[dev];
  }
  if (ws == nullptr) {  // no call on this device yet: nothing to report
    *status_out = 0;
    return DSAI_OK;
  }
  return dsai_read_status(ws, stream, status_out);
}
