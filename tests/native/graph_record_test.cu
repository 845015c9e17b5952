// Host-only test of the launch recorder (csrc/graph.h): while a recorder is
// active, launch_kernel() records the kernel, its configuration and a copy
// of its argument values, and launches nothing.  Built by
// tests/test_graph_record.py with nvcc and run on the host; no CUDA call is
// made, so it needs no GPU.
#include <cstdio>
#include <cstring>

#include "graph.h"

struct alignas(64) BigArg {  // a tensor-map-like 128-B, 64-B aligned argument
  unsigned char bytes[128];
};

struct Params {
  const float* p;
  int n;
  long long x;
};

__global__ void kernel_a(BigArg m, Params prm, int k) {}
__global__ void kernel_b(const int* a, int* b, int n) {}

#define CHECK(c)                                              \
  do {                                                        \
    if (!(c)) {                                               \
      std::printf("FAILED line %d: %s\n", __LINE__, #c);      \
      return 1;                                               \
    }                                                         \
  } while (0)

int main() {
  using namespace dsai;
  CHECK(active_recorder() == nullptr);
  static LaunchRecorder rec;
  BigArg m;
  for (int i = 0; i < 128; ++i) m.bytes[i] = static_cast<unsigned char>(i * 7 + 1);
  Params prm{reinterpret_cast<const float*>(0x1234560), 77, -5};
  cudaLaunchAttribute attr[2];
  std::memset(attr, 0xAB, sizeof(attr));  // unused union bytes left as garbage, as launchers do
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(296);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = 114688;
  cfg.stream = reinterpret_cast<cudaStream_t>(0x99);
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  {
    RecordScope scope(&rec);
    CHECK(active_recorder() == &rec);
    CHECK(launch_kernel(cfg, kernel_a, m, prm, 3) == cudaSuccess);
    cudaLaunchConfig_t c2 = {};
    c2.gridDim = dim3(64);
    c2.blockDim = dim3(1024);
    const int* a = reinterpret_cast<const int*>(0x1000);
    int* b = reinterpret_cast<int*>(0x2000);
    short n = 9;  // converted to the kernel's int parameter
    CHECK(launch_kernel(c2, kernel_b, a, b, n) == cudaSuccess);
  }
  CHECK(active_recorder() == nullptr);
  CHECK(rec.n == 2 && !rec.overflow);

  const KernelRecord& r0 = rec.recs[0];
  CHECK(r0.func == reinterpret_cast<const void*>(kernel_a));
  CHECK(r0.grid.x == 296 && r0.block.x == 192 && r0.smem == 114688);
  CHECK(r0.nattrs == 2);
  CHECK(r0.attrs[0].id == cudaLaunchAttributeProgrammaticStreamSerialization);
  CHECK(r0.attrs[1].id == cudaLaunchAttributeClusterDimension && r0.attrs[1].val.clusterDim.x == 2);
  CHECK(r0.nargs == 3);
  CHECK(r0.arg_off[0] % 64 == 0);  // the 64-B aligned argument stays aligned
  CHECK(std::memcmp(r0.args + r0.arg_off[0], &m, sizeof(m)) == 0);
  CHECK(r0.arg_off[1] % alignof(Params) == 0);
  Params back;
  std::memcpy(&back, r0.args + r0.arg_off[1], sizeof(back));
  CHECK(back.p == prm.p && back.n == 77 && back.x == -5);
  int k = 0;
  std::memcpy(&k, r0.args + r0.arg_off[2], sizeof(k));
  CHECK(k == 3);
  CHECK(reinterpret_cast<uintptr_t>(r0.args) % 64 == 0);

  const KernelRecord& r1 = rec.recs[1];
  CHECK(r1.func == reinterpret_cast<const void*>(kernel_b) && r1.nargs == 3 && r1.nattrs == 0);
  CHECK(r1.grid.x == 64 && r1.block.x == 1024 && r1.smem == 0);
  const int* a2 = nullptr;
  std::memcpy(&a2, r1.args + r1.arg_off[0], sizeof(a2));
  CHECK(a2 == reinterpret_cast<const int*>(0x1000));
  int n2 = 0;
  std::memcpy(&n2, r1.args + r1.arg_off[2], sizeof(n2));
  CHECK(n2 == 9);

  // More launches than a record holds: flagged, not written past the end.
  static LaunchRecorder full;
  {
    RecordScope scope(&full);
    for (int i = 0; i < kRecMaxKernels; ++i) CHECK(launch_kernel(cfg, kernel_a, m, prm, i) == cudaSuccess);
    CHECK(launch_kernel(cfg, kernel_a, m, prm, 99) == cudaErrorNotSupported);
  }
  CHECK(full.n == kRecMaxKernels && full.overflow);
  // Nested scopes restore the outer recorder.
  {
    RecordScope outer(&rec);
    {
      RecordScope inner(&full);
      CHECK(active_recorder() == &full);
    }
    CHECK(active_recorder() == &rec);
  }
  std::printf("ok\n");
  return 0;
}
