"""Drop-in entry point of the DSA top-K indexer.

``kernel(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table,
topk_indices)`` has the signature, argument meaning and destination-passing
style of the reference's ``solution/python/solution.py::kernel``
(solution/python/solution.py:25-26, config.toml:6-9) and fails the same way:
a ``RuntimeError`` for a tensor that is not CUDA / contiguous / of the
expected dtype or shape (the reference's TORCH_CHECKs,
solution/python/kernel.cu:1227-1240, :1273-1279).

Everything runs in ``libdsai.so`` on the caller's current CUDA stream, with
no host synchronisation.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

__all__ = ["kernel", "run", "run_pairs", "merge_pairs", "read_status", "write_index_k", "IndexerGraph",
           "sparse_attention", "read_attn_status"]

_FP8 = getattr(torch, "float8_e4m3fn", None)
# Per-call host work is most of the cost of a small call: the current device
# and the raw stream handle are read without building torch.cuda objects.
_current_device = torch._C._cuda_getDevice
_current_raw_stream = torch._C._cuda_getCurrentRawStream
# DSAI_GRAPH=1 in the environment (read once) makes kernel() launch through
# the library's graph cache, as run(..., graph=True) does.  Off by default:
# replays cut the host work per call but give up the programmatic overlap of
# one call's first kernel with the previous call's last.
_KERNEL_GRAPH = os.environ.get("DSAI_GRAPH", "0") == "1"


def _call_on(dev_index: int, fn, *args) -> int:
    """Calls fn(*args) with `dev_index` as the current CUDA device."""
    if _current_device() == dev_index:
        return fn(*args)
    with torch.cuda.device(dev_index):
        return fn(*args)


def _req(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_int32(t: torch.Tensor, name: str) -> None:
    _req(t.is_cuda and t.is_contiguous() and t.dtype == torch.int32,
         f"{name} must be int32 contiguous CUDA")


def _check_scoring_inputs(q, k, w, rows: int) -> None:
    _req(q.is_cuda and q.is_contiguous(), "q_index_fp8 must be contiguous CUDA")
    _req(k.is_cuda and k.is_contiguous(), "k_index_cache_fp8 must be contiguous CUDA")
    _req(w.is_cuda and w.is_contiguous() and w.dtype == torch.float32,
         "weights must be float32 contiguous CUDA")
    _req(q.dtype in (_FP8, torch.uint8, torch.int8), "q_index_fp8 must be float8_e4m3fn")
    _req(q.numel() == rows * _lib.NUM_HEADS * _lib.HEAD_DIM, "q_index_fp8 shape must be [B, 64, 128]")
    _req(k.element_size() == 1 and k.numel() % _lib.PAGE_BYTES == 0,
         "k_index_cache_fp8 must be uint8 [num_pages, 64, 1, 132]")
    _req(w.numel() == rows * _lib.NUM_HEADS, "weights shape must be [B, 64]")


def _args(q, k, w, seq_lens, block_table, out, logits_out, flags: int, rows_per_seq: int = 1) -> _lib.DsaiArgs:
    rows, max_pages = int(block_table.size(0)), int(block_table.size(1))
    a = _lib.DsaiArgs()
    a.q = q.data_ptr() if q is not None else None
    a.k_cache = k.data_ptr() if k is not None else None
    a.weights = w.data_ptr() if w is not None else None
    a.seq_lens = seq_lens.data_ptr()
    a.block_table = block_table.data_ptr()
    a.topk_indices = out.data_ptr() if out is not None else None
    a.logits_out = logits_out.data_ptr() if logits_out is not None else None
    a.rows = rows
    a.max_pages = max_pages
    a.num_pages = (k.numel() // _lib.PAGE_BYTES) if k is not None else 0
    a.flags = flags
    a.ev_after_score = None
    a.rows_per_seq = rows_per_seq
    return a


def run(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices,
        logits_out: torch.Tensor | None = None, score_all_rows: bool = False,
        event_after_score: torch.cuda.Event | None = None, workspace: "_lib.Workspace | None" = None,
        rows_per_seq: int = 1, graph: bool = False):
    """The indexer with optional extras: ``logits_out`` ([B, max_pages*64]
    fp32) receives the scored logits (entries at t >= seq_len are left
    untouched; rows with seq_len <= 2048 are scored only with
    ``score_all_rows``), ``event_after_score`` is recorded between the
    scoring and the selection launches.  ``rows_per_seq`` = 2..4 declares
    consecutive groups of that many rows to be query tokens of one sequence
    (multi-query decode, next-n / MTP, causal prefill rows) that agree on
    ``block_table`` over every page each of them reaches: each group's K
    pages are then read once, through the block-table row of its longest
    row.  The results are those of independent rows.  ``graph`` launches the
    call's kernels as one CUDA graph from the library's cache of executable
    graphs (one per device, stream and launch plan; the call's pointers are
    written into the cached graph's kernel nodes, nothing is re-captured):
    the reference's replay of every call from a graph cache
    (solution/python/kernel.cu:1101-1199)."""
    _check_int32(block_table, "block_table")
    _check_int32(seq_lens, "seq_lens")
    _check_int32(topk_indices, "topk_indices")
    rows, max_pages = int(block_table.size(0)), int(block_table.size(1))
    _req(topk_indices.dim() == 2 and topk_indices.size(0) == rows and topk_indices.size(1) == _lib.TOPK,
         "topk_indices shape must be [B, 2048]")
    _req(seq_lens.numel() == rows, "seq_lens shape must be [B]")
    _req(isinstance(rows_per_seq, int) and 1 <= rows_per_seq <= 4, "rows_per_seq must be 1 to 4")
    _req(rows % rows_per_seq == 0, "rows must be a multiple of rows_per_seq")
    if rows == 0:
        return
    lib = _lib.load_library()
    needs_scoring = max_pages * _lib.PAGE_SIZE > _lib.TOPK or score_all_rows
    if needs_scoring:
        _check_scoring_inputs(q_index_fp8, k_index_cache_fp8, weights, rows)
    if logits_out is not None:
        _req(logits_out.is_cuda and logits_out.is_contiguous() and logits_out.dtype == torch.float32
             and logits_out.numel() == rows * max_pages * _lib.PAGE_SIZE,
             "logits_out must be float32 contiguous CUDA [B, max_pages*64]")
    dev = block_table.device
    idx = dev.index
    stream = _current_raw_stream(idx)
    ws = workspace or _lib.default_workspace(dev, stream)
    ws_ptr, ws_bytes = ws.get(rows, max_pages, stream)
    a = _args(q_index_fp8 if needs_scoring else None, k_index_cache_fp8 if needs_scoring else None,
              weights if needs_scoring else None, seq_lens, block_table, topk_indices, logits_out,
              (_lib.FLAG_SCORE_ALL_ROWS if score_all_rows else 0) | (_lib.FLAG_GRAPH if graph else 0),
              rows_per_seq)
    if needs_scoring:
        a.num_pages = k_index_cache_fp8.numel() // _lib.PAGE_BYTES
    if event_after_score is not None:
        a.ev_after_score = event_after_score.cuda_event
    _lib.check(_call_on(idx, lib.dsai_run, ctypes.byref(a), ws_ptr, ws_bytes, stream))


def kernel(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices):
    """Drop-in for the reference's ``solution.py::kernel``: writes the top-2048
    physical slot ids of every row into ``topk_indices`` ([B, 2048] int32,
    -1 padded) and returns None."""
    run(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices, graph=_KERNEL_GRAPH)


def run_pairs(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, token_offset: int,
              out_scores: torch.Tensor, out_tokens: torch.Tensor,
              workspace: "_lib.Workspace | None" = None):
    """Per-row top-2048 (fp32 score, token + token_offset) pairs — the local
    half of a page-range split of long rows across GPUs."""
    _check_int32(block_table, "block_table")
    _check_int32(seq_lens, "seq_lens")
    rows, max_pages = int(block_table.size(0)), int(block_table.size(1))
    _req(out_scores.is_cuda and out_scores.dtype == torch.float32 and out_scores.is_contiguous()
         and out_scores.numel() == rows * _lib.TOPK, "out_scores must be float32 [B, 2048]")
    _check_int32(out_tokens, "out_tokens")
    _req(out_tokens.numel() == rows * _lib.TOPK, "out_tokens must be int32 [B, 2048]")
    if rows == 0:
        return
    _check_scoring_inputs(q_index_fp8, k_index_cache_fp8, weights, rows)
    lib = _lib.load_library()
    dev = block_table.device
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws = workspace or _lib.default_workspace(dev, stream)
    ws_ptr, ws_bytes = ws.get(rows, max_pages, stream)
    a = _args(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, None, None, 0)
    with torch.cuda.device(dev):
        _lib.check(lib.dsai_run_pairs(ctypes.byref(a), int(token_offset), out_scores.data_ptr(),
                                      out_tokens.data_ptr(), ws_ptr, ws_bytes, stream))


def merge_pairs(scores: torch.Tensor, tokens: torch.Tensor, block_table_row: torch.Tensor,
                seq_len: torch.Tensor, out: torch.Tensor):
    """Top-2048 physical ids of ONE row from (score, token) candidates
    gathered from several partial rows (token -1 = padding)."""
    _req(scores.is_cuda and scores.dtype == torch.float32 and scores.is_contiguous(),
         "scores must be float32 contiguous CUDA")
    _check_int32(tokens, "tokens")
    _check_int32(block_table_row, "block_table_row")
    _check_int32(seq_len, "seq_len")
    _check_int32(out, "out")
    _req(scores.numel() == tokens.numel(), "scores and tokens must have the same length")
    _req(out.numel() == _lib.TOPK, "out must hold 2048 int32")
    lib = _lib.load_library()
    dev = out.device
    stream = torch.cuda.current_stream(dev).cuda_stream
    with torch.cuda.device(dev):
        _lib.check(lib.dsai_merge_pairs(scores.data_ptr(), tokens.data_ptr(), int(scores.numel()),
                                        block_table_row.data_ptr(), int(block_table_row.numel()),
                                        seq_len.data_ptr(), out.data_ptr(), stream))


def write_index_k(k_new: torch.Tensor, slot_ids: torch.Tensor, k_index_cache_fp8: torch.Tensor) -> None:
    """Index-K cache writer (the step before the indexer in a decode step):
    quantises the new keys ``k_new`` ([n, 128] float32 or bfloat16) to e4m3
    with one fp32 scale per token (max |k| / 448) and stores token i at
    physical slot id ``slot_ids[i]`` (int32 page*64 + slot, -1 = skip) of
    ``k_index_cache_fp8`` ([num_pages, 64, 1, 132] uint8), in the page layout
    ``kernel`` reads.  Runs on the current stream; no host synchronisation."""
    _req(k_new.is_cuda and k_new.is_contiguous() and k_new.dtype in (torch.float32, torch.bfloat16),
         "k_new must be float32 or bfloat16 contiguous CUDA")
    _req(k_new.dim() == 2 and k_new.size(1) == _lib.HEAD_DIM, "k_new shape must be [n, 128]")
    _check_int32(slot_ids, "slot_ids")
    _req(slot_ids.numel() == k_new.size(0), "slot_ids must hold one id per new token")
    _req(k_index_cache_fp8.is_cuda and k_index_cache_fp8.is_contiguous()
         and k_index_cache_fp8.element_size() == 1 and k_index_cache_fp8.numel() % _lib.PAGE_BYTES == 0,
         "k_index_cache_fp8 must be uint8 contiguous CUDA [num_pages, 64, 1, 132]")
    n = int(k_new.size(0))
    if n == 0:
        return
    lib = _lib.load_library()
    dev = k_new.device
    dtype = _lib.DTYPE_BF16 if k_new.dtype == torch.bfloat16 else _lib.DTYPE_F32
    with torch.cuda.device(dev):
        _lib.check(lib.dsai_write_k(k_new.data_ptr(), dtype, slot_ids.data_ptr(), n,
                                    k_index_cache_fp8.data_ptr(),
                                    int(k_index_cache_fp8.numel() // _lib.PAGE_BYTES),
                                    torch.cuda.current_stream(dev).cuda_stream))


_attn_ws: dict = {}


def _attn_workspace(dev: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Workspace of the sparse attention per (device, stream), so calls on
    different streams never share one (status header zeroed once at
    allocation; grown when a call needs more)."""
    key = (dev.index, int(stream))
    ws = _attn_ws.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=dev)
        _attn_ws[key] = ws
    return ws


def sparse_attention(q_nope: torch.Tensor, q_pe: torch.Tensor, ckv_cache: torch.Tensor, kpe_cache: torch.Tensor,
                     sparse_indices: torch.Tensor, sm_scale: float, output: torch.Tensor, lse: torch.Tensor) -> None:
    """Sparse MLA attention over the indexer's top-2048 slots (the operator
    after the indexer in a DSA decode step), destination-passing: for token
    t and head h over the entries of ``sparse_indices[t]`` that are not -1
    (flat slot ids page*64 + slot), ``output[t, h]`` ([T, 16, 512] bf16)
    gets softmax(scores * sm_scale) @ ckv and ``lse[t, h]`` ([T, 16] fp32)
    the base-2 log-sum-exp of the scaled scores (0 and -inf for a token
    with no valid entry).  q_nope [T, 16, 512], q_pe [T, 16, 64],
    ckv_cache [num_pages, 64, 512] and kpe_cache [num_pages, 64, 64] are
    bf16.  Runs on the current stream."""
    bf = torch.bfloat16
    for name, x in (("q_nope", q_nope), ("q_pe", q_pe), ("ckv_cache", ckv_cache), ("kpe_cache", kpe_cache),
                    ("output", output)):
        _req(x.is_cuda and x.is_contiguous() and x.dtype == bf, f"{name} must be bfloat16 contiguous CUDA")
    _check_int32(sparse_indices, "sparse_indices")
    _req(lse.is_cuda and lse.is_contiguous() and lse.dtype == torch.float32, "lse must be float32 contiguous CUDA")
    T = int(q_nope.size(0)) if q_nope.dim() == 3 else -1
    H, D, DP = _lib.ATTN_HEADS, _lib.ATTN_CKV_DIM, _lib.ATTN_KPE_DIM
    _req(q_nope.dim() == 3 and tuple(q_nope.shape[1:]) == (H, D), "q_nope shape must be [T, 16, 512]")
    _req(tuple(q_pe.shape) == (T, H, DP), "q_pe shape must be [T, 16, 64]")
    _req(ckv_cache.dim() == 3 and tuple(ckv_cache.shape[1:]) == (_lib.PAGE_SIZE, D),
         "ckv_cache shape must be [num_pages, 64, 512]")
    num_pages = int(ckv_cache.size(0))
    _req(tuple(kpe_cache.shape) == (num_pages, _lib.PAGE_SIZE, DP), "kpe_cache shape must be [num_pages, 64, 64]")
    _req(tuple(sparse_indices.shape) == (T, _lib.TOPK), "sparse_indices shape must be [T, 2048]")
    _req(tuple(output.shape) == (T, H, D) and tuple(lse.shape) == (T, H), "output / lse shapes must be [T, 16, 512] / [T, 16]")
    if T == 0:
        return
    lib = _lib.load_library()
    dev = q_nope.device
    with torch.cuda.device(dev):
        stream = torch.cuda.current_stream(dev).cuda_stream
        ws = _attn_workspace(dev, stream, int(lib.dsai_sparse_attn_workspace_size(T)))
        a = _lib.DsaiAttnArgs()
        a.q_nope, a.q_pe = q_nope.data_ptr(), q_pe.data_ptr()
        a.ckv_cache, a.kpe_cache = ckv_cache.data_ptr(), kpe_cache.data_ptr()
        a.sparse_indices = sparse_indices.data_ptr()
        a.output, a.lse = output.data_ptr(), lse.data_ptr()
        a.sm_scale = float(sm_scale)
        a.num_tokens, a.num_pages = T, num_pages
        _lib.check(lib.dsai_sparse_attn(ctypes.byref(a), ws.data_ptr(), ws.numel(), stream))


def read_attn_status(device=None) -> int:
    """Returns and clears the status bits of the sparse attention's workspace
    of `device` and its current stream (synchronises that stream)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    ws = _attn_ws.get((dev.index, torch.cuda.current_stream(dev).cuda_stream))
    if ws is None:
        return 0
    lib = _lib.load_library()
    v = ctypes.c_int32(0)
    with torch.cuda.device(dev):
        _lib.check(lib.dsai_read_status(ws.data_ptr(), torch.cuda.current_stream(dev).cuda_stream, ctypes.byref(v)))
    return int(v.value)


def read_status(device=None) -> int:
    """Returns and clears the device status bits of the default workspace of
    `device` and its current stream, the one ``kernel()`` used when called
    on that stream (synchronises the stream)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev).cuda_stream
    ws = _lib.default_workspace(dev, stream)
    return ws.read_status(stream)


class IndexerGraph:
    """One indexer call on fixed tensors, captured once in a CUDA graph and
    replayed (the reference's graph cache, solution/python/kernel.cu:1101-1199,
    as an explicit object: no key lookup per call).

    The graph holds the addresses of the six tensors given here and of a
    workspace of its own: refresh their contents in place (``copy_``) between
    replays; shapes and addresses are fixed.  ``replay()`` launches the two
    kernels on the current stream with one graph launch, which removes the
    per-call host work of ``kernel()`` (argument checks, ctypes call, two
    launches) that dominates on small batches.  ``rows_per_seq`` is that of
    ``run``."""

    def __init__(self, q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices,
                 rows_per_seq: int = 1):
        self.tensors = (q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices)
        self.rows_per_seq = rows_per_seq
        dev = block_table.device
        self.workspace = _lib.Workspace(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            # sizes the workspace, encodes the tensor maps, sets kernel attributes
            run(*self.tensors, workspace=self.workspace, rows_per_seq=rows_per_seq)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, capture_error_mode="thread_local"):
            run(*self.tensors, workspace=self.workspace, rows_per_seq=rows_per_seq)

    def replay(self) -> None:
        """Runs the captured call on the current stream."""
        self.graph.replay()
