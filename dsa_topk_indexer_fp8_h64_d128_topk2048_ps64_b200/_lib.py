"""ctypes binding of ``libdsai.so`` (the C ABI in ``include/dsai.h``).

There is no fallback: if the library is missing or fails to load, importing
the operator raises, and every call goes to the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libdsai.so"

NUM_HEADS = 64
HEAD_DIM = 128
PAGE_SIZE = 64
TOPK = 2048
PAGE_BYTES = 8448
SCALE_OFFSET = 8192

DSAI_OK = 0
STATUS_SEQLEN_CLAMPED = 0x1
STATUS_BAD_PAGE = 0x2
STATUS_WAIT_TIMEOUT = 0x4
STATUS_BAD_INDEX = 0x8
ATTN_HEADS = 16
ATTN_CKV_DIM = 512
ATTN_KPE_DIM = 64
FLAG_SCORE_ALL_ROWS = 0x1
FLAG_GRAPH = 0x2
DTYPE_F32 = 0
DTYPE_BF16 = 1
E_INVALID = -1      # DSAI_E_* return codes
E_WORKSPACE = -2
E_CUDA = -3
E_UNSUPPORTED = -4

EXPORTED_SYMBOLS = (
    "dsai_workspace_size", "dsai_workspace_init", "dsai_run", "dsai_run_pairs",
    "dsai_merge_pairs", "dsai_read_status", "dsai_last_error", "dsai_version",
    "dsai_run_noalloc", "dsai_noalloc_read_status", "dsai_selftest_wait_timeout", "dsai_write_k",
    "dsai_sparse_attn_workspace_size", "dsai_sparse_attn", "dsai_graph_cache_entries",
)


class DsaiArgs(ctypes.Structure):
    """Mirror of ``dsai_args`` in include/dsai.h."""
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k_cache", ctypes.c_void_p),
        ("weights", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("block_table", ctypes.c_void_p),
        ("topk_indices", ctypes.c_void_p),
        ("logits_out", ctypes.c_void_p),
        ("rows", ctypes.c_int32),
        ("max_pages", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
        ("flags", ctypes.c_int32),
        ("ev_after_score", ctypes.c_void_p),
        ("rows_per_seq", ctypes.c_int32),
    ]


class DsaiAttnArgs(ctypes.Structure):
    """Mirror of ``dsai_attn_args`` in include/dsai.h."""
    _fields_ = [
        ("q_nope", ctypes.c_void_p),
        ("q_pe", ctypes.c_void_p),
        ("ckv_cache", ctypes.c_void_p),
        ("kpe_cache", ctypes.c_void_p),
        ("sparse_indices", ctypes.c_void_p),
        ("output", ctypes.c_void_p),
        ("lse", ctypes.c_void_p),
        ("sm_scale", ctypes.c_float),
        ("num_tokens", ctypes.c_int32),
        ("num_pages", ctypes.c_int32),
    ]


_lib = None
_lib_lock = threading.Lock()


def load_library(path: Path | None = None) -> ctypes.CDLL:
    """Loads libdsai.so once; raises if it is missing."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise RuntimeError(
                f"{p} is missing: build it with `python -m "
                "dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200.build` (needs nvcc)")
        lib = ctypes.CDLL(str(p))
        vp, i32, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_size_t
        lib.dsai_workspace_size.argtypes = [i32, i32]
        lib.dsai_workspace_size.restype = sz
        lib.dsai_workspace_init.argtypes = [vp, sz, vp]
        lib.dsai_workspace_init.restype = ctypes.c_int
        lib.dsai_run.argtypes = [ctypes.POINTER(DsaiArgs), vp, sz, vp]
        lib.dsai_run.restype = ctypes.c_int
        lib.dsai_run_pairs.argtypes = [ctypes.POINTER(DsaiArgs), i32, vp, vp, vp, sz, vp]
        lib.dsai_run_pairs.restype = ctypes.c_int
        lib.dsai_merge_pairs.argtypes = [vp, vp, i32, vp, i32, vp, vp, vp]
        lib.dsai_merge_pairs.restype = ctypes.c_int
        lib.dsai_run_noalloc.argtypes = [ctypes.POINTER(DsaiArgs), vp]
        lib.dsai_run_noalloc.restype = ctypes.c_int
        lib.dsai_noalloc_read_status.argtypes = [vp, ctypes.POINTER(i32)]
        lib.dsai_noalloc_read_status.restype = ctypes.c_int
        lib.dsai_selftest_wait_timeout.argtypes = [vp, ctypes.c_uint64, vp]
        lib.dsai_selftest_wait_timeout.restype = ctypes.c_int
        lib.dsai_write_k.argtypes = [vp, i32, vp, i32, vp, i32, vp]
        lib.dsai_write_k.restype = ctypes.c_int
        lib.dsai_sparse_attn_workspace_size.argtypes = [i32]
        lib.dsai_sparse_attn_workspace_size.restype = sz
        lib.dsai_sparse_attn.argtypes = [ctypes.POINTER(DsaiAttnArgs), vp, sz, vp]
        lib.dsai_sparse_attn.restype = ctypes.c_int
        lib.dsai_read_status.argtypes = [vp, vp, ctypes.POINTER(i32)]
        lib.dsai_read_status.restype = ctypes.c_int
        lib.dsai_last_error.argtypes = []
        lib.dsai_last_error.restype = ctypes.c_char_p
        lib.dsai_version.argtypes = []
        lib.dsai_version.restype = ctypes.c_char_p
        lib.dsai_graph_cache_entries.argtypes = []
        lib.dsai_graph_cache_entries.restype = ctypes.c_int
        _lib = lib
        return lib


def check(rc: int) -> None:
    if rc != DSAI_OK:
        msg = load_library().dsai_last_error().decode(errors="replace")
        raise RuntimeError(f"dsai error {rc}: {msg}")


def workspace_size(rows: int, max_pages: int) -> int:
    return int(load_library().dsai_workspace_size(rows, max_pages))


class Workspace:
    """A device workspace for dsai_run, grown on demand.  Use one per
    stream: two calls in flight on one workspace at once corrupt each
    other.  Its header holds the sticky device status word."""

    def __init__(self, device: torch.device):
        self.device = torch.device(device)
        self.buf: torch.Tensor | None = None
        self._shape = None      # (rows, max_pages) of the last get()
        self._span = (0, 0)     # (pointer, bytes) it returned

    def get(self, rows: int, max_pages: int, stream: int) -> tuple[int, int]:
        if self._shape == (rows, max_pages) and self.buf is not None:
            return self._span
        need = workspace_size(rows, max_pages)
        if self.buf is None or self.buf.numel() < need:
            size = max(need, 1 << 20)
            if self.buf is not None:
                size = max(size, 2 * self.buf.numel())
            self.buf = torch.empty(size, dtype=torch.uint8, device=self.device)
            check(load_library().dsai_workspace_init(self.buf.data_ptr(), self.buf.numel(), stream))
        self._shape = (rows, max_pages)
        self._span = (self.buf.data_ptr(), self.buf.numel())
        return self._span

    def read_status(self, stream: int) -> int:
        """Returns and clears the device status bits (synchronises `stream`)."""
        if self.buf is None:
            return 0
        out = ctypes.c_int32(0)
        check(load_library().dsai_read_status(self.buf.data_ptr(), stream, ctypes.byref(out)))
        return int(out.value)


_workspaces: dict[tuple[int, int], Workspace] = {}
_workspaces_lock = threading.Lock()


def default_workspace(device: torch.device, stream: int | None = None) -> Workspace:
    """The workspace that ``kernel()`` / ``run()`` use on `device` when
    called on `stream` (a raw ``cudaStream_t`` value; None = the device's
    current torch stream).  One workspace per (device, stream): calls
    issued on different streams may overlap on the GPU, and a shared
    workspace would let them overwrite each other's histograms, counters
    and logits.  Calls on one stream are ordered, so they share one."""
    idx = torch.device(device).index
    if idx is None:
        idx = torch.cuda.current_device()
    if stream is None:
        stream = torch.cuda.current_stream(idx).cuda_stream
    key = (idx, int(stream))
    ws = _workspaces.get(key)
    if ws is None:
        with _workspaces_lock:
            ws = _workspaces.get(key)
            if ws is None:
                ws = _workspaces[key] = Workspace(torch.device("cuda", idx))
    return ws
