"""Builds the reference's active CUDA path (solution/python/kernel.cu, the
kernel its solution.py::kernel JIT-compiles) for timing beside ours.

As shipped it does not build with nvcc 12.9: two stage-1 kernels
(paged_mqa_logits_umma_kernel_persistent and _persistent_ws) declare their
3-stage K ring, 3 x 16 KB, as static shared memory, which puts them above
the 48 KB static limit (59,152 and 59,200 B).  The reference was built with
CUDA 13.2.  This script makes the one change needed and nothing else:

  1. both declarations
         __shared__ __align__(1024) __nv_fp8_e4m3 smem_k[kKVStages][kUMMA_M * kHeadDim];
     become a reference of the same type and extent into dynamic shared
     memory (1024-B aligned inside a 49,152 + 1,024 B dynamic buffer);
  2. the two launches of those kernels pass that dynamic size instead of 0;
  3. the host entry point sets cudaFuncAttributeMaxDynamicSharedMemorySize
     for both kernels once, before its graph capture.

Every other line (the kernels' arithmetic, the radix top-K, the fast path,
the graph cache) is the reference's.  The patched source is written to a
temporary directory only; the extension (built with the reference's own
flags, as its solution.py does) is copied to
baseline/_ref/dsa_topk_indexer_ref_active*.so.  Run where the reference
checkout is present:  python baseline/build_active_variant.py
"""
from __future__ import annotations

import shutil
import sys
import tempfile
from pathlib import Path

REF = Path("/root/reference/solution/python")
OUT_DIR = Path(__file__).resolve().parent / "_ref"
NAME = "dsa_topk_indexer_ref_active"

DECL = "    __shared__ __align__(1024) __nv_fp8_e4m3 smem_k[kKVStages][kUMMA_M * kHeadDim];\n"
DYN_DECL = (
    "    extern __shared__ __align__(1024) unsigned char dsa_dyn_smem_k[];\n"
    "    auto& smem_k = *reinterpret_cast<__nv_fp8_e4m3 (*)[kKVStages][kUMMA_M * kHeadDim]>(\n"
    "        dsa_dyn_smem_k + ((1024u - (static_cast<unsigned>(reinterpret_cast<uintptr_t>(dsa_dyn_smem_k)) & 1023u)) & 1023u));\n"
)
STAGES = "constexpr int kKVStages = 3;\n"
STAGES_NEW = STAGES + "constexpr int kDynSmemK = kKVStages * 128 * kHeadDim + 1024;\n"
LAUNCHES = [
    ("paged_mqa_logits_umma_kernel_persistent_ws<<<grid, block, 0, s>>>(",
     "paged_mqa_logits_umma_kernel_persistent_ws<<<grid, block, kDynSmemK, s>>>("),
    ("paged_mqa_logits_umma_kernel_persistent<<<grid, block, 0, s>>>(",
     "paged_mqa_logits_umma_kernel_persistent<<<grid, block, kDynSmemK, s>>>("),
]
ENTRY = """    torch::Tensor topk_indices)
{
"""
ENTRY_NEW = ENTRY + """    static std::once_flag dsa_dyn_smem_once;
    std::call_once(dsa_dyn_smem_once, [] {
        cudaFuncSetAttribute(paged_mqa_logits_umma_kernel_persistent_ws,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmemK);
        cudaFuncSetAttribute(paged_mqa_logits_umma_kernel_persistent,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmemK);
    });
"""


def patched_source() -> str:
    src = (REF / "kernel.cu").read_text()

    def once(text, old, new, count=1):
        n = text.count(old)
        if n != count:
            raise RuntimeError(f"expected {count} occurrence(s) of {old[:60]!r}, found {n}")
        return text.replace(old, new)

    src = once(src, DECL, DYN_DECL, count=2)
    src = once(src, STAGES, STAGES_NEW)
    for old, new in LAUNCHES:
        src = once(src, old, new)
    src = once(src, ENTRY, ENTRY_NEW)
    return src


def build() -> Path:
    import torch.utils.cpp_extension as ext
    OUT_DIR.mkdir(exist_ok=True)
    with tempfile.TemporaryDirectory() as tmp:
        cu = Path(tmp) / "kernel.cu"
        cu.write_text(patched_source())
        bdir = Path(tmp) / "build"
        bdir.mkdir()
        mod = ext.load(name=NAME, sources=[str(cu)],
                       extra_cuda_cflags=["-O3", "--expt-relaxed-constexpr",
                                          "-gencode", "arch=compute_100a,code=sm_100a"],
                       extra_include_paths=[str(REF)], build_directory=str(bdir), verbose=False)
        so = Path(mod.__file__)
        dst = OUT_DIR / so.name
        shutil.copy2(so, dst)
    return dst


if __name__ == "__main__":
    if not (REF / "kernel.cu").exists():
        sys.exit("the reference checkout is not present")
    print(build())
