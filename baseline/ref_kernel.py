"""Loader of the reference's own sm_100a indexer kernel.

``baseline/_ref/libref_tvm_indexer.so`` is built by ``make -C baseline``
from the reference's TVM-FFI variant (solution/cuda/kernel.cu, unmodified)
and exports the reference's entry point ``kernel`` (solution/cuda/
kernel.cu:507).  It is called here exactly as the reference's harness calls
it: through tvm_ffi with the six torch tensors, on torch's current stream
(the reference takes the stream and its fp16 logits scratch from the tvm_ffi
environment, solution/cuda/kernel.cu:471-479).

This module is measurement and test infrastructure: the golden-vector
script, the parity tests and bench.py's ``reference_kernel`` key use it;
the package never does.
"""
from __future__ import annotations

from pathlib import Path

LIB = Path(__file__).resolve().parent / "_ref" / "libref_tvm_indexer.so"
SOURCE = "solution/cuda/kernel.cu (TVM-FFI variant, unmodified)"
ACTIVE_NAME = "dsa_topk_indexer_ref_active"
ACTIVE_SOURCE = ("solution/python/kernel.cu (the active path; static K ring moved to dynamic shared "
                 "memory to build with nvcc 12.9, baseline/build_active_variant.py)")

_fn = None
_active = None


def available() -> tuple[bool, str]:
    """(True, "") if the library is built and tvm_ffi imports, else (False, why)."""
    if not LIB.exists():
        return False, f"{LIB.name} not built (make -C baseline needs the reference checkout)"
    try:
        import tvm_ffi  # noqa: F401
    except Exception as e:  # pragma: no cover - depends on the image
        return False, f"tvm_ffi unavailable: {e}"
    return True, ""


def load():
    """The reference's `kernel(q, k_cache, weights, seq_lens, block_table,
    topk_indices)` (destination-passing, returns None)."""
    global _fn
    if _fn is None:
        ok, why = available()
        if not ok:
            raise RuntimeError(why)
        import tvm_ffi
        mod = tvm_ffi.load_module(str(LIB))
        _fn = mod["kernel"]
    return _fn


def kernel(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices) -> None:
    """Calls the reference kernel on torch's current stream."""
    load()(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices)


def active_lib() -> Path | None:
    hits = sorted((Path(__file__).resolve().parent / "_ref").glob(ACTIVE_NAME + "*.so"))
    return hits[0] if hits else None


def active_available() -> tuple[bool, str]:
    if active_lib() is None:
        return False, "active variant not built (python baseline/build_active_variant.py needs the reference checkout)"
    return True, ""


def active_kernel(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices) -> None:
    """The reference's active path: its torch extension's `run`, which
    solution/python/solution.py::kernel forwards to (solution.py:25-26)."""
    global _active
    if _active is None:
        import importlib.machinery
        import importlib.util
        import torch  # noqa: F401  (the extension links against torch)
        so = active_lib()
        if so is None:
            raise RuntimeError(active_available()[1])
        loader = importlib.machinery.ExtensionFileLoader(ACTIVE_NAME, str(so))
        spec = importlib.util.spec_from_file_location(ACTIVE_NAME, str(so), loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _active = mod
    _active.run(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices)
