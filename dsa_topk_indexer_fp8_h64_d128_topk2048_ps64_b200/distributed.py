"""Multi-GPU layer: one process per GPU (torch.distributed, NCCL over
NVLink/NVSwitch), used only where the indexer shards naturally.

* Rows are independent (batched decode): ``shard_rows`` gives each rank a
  contiguous block of rows, balanced by their token counts; each rank runs the
  indexer on its rows with its own K pool.  No collective is on the data path;
  ``gather_rows`` optionally assembles every rank's output on all ranks.
* One very long row (a single long request) is split by page range:
  ``split_row_topk`` scores the rank's pages as a sub-row, selects its local
  top-2048 as (fp32 score, global token) pairs, exchanges the 2048 pairs of
  every rank with one all-gather (scores and tokens packed together, 16 KB
  per rank) and merges them into the
  row's top-2048 physical ids with the full block table.

The reference is single-GPU; this layer has no counterpart there.  The local
compute and merge steps are parameters so the host logic (page ranges, token
offsets, the exchange) can be exercised on CPU ranks with any implementation;
on GPUs the defaults are the CUDA entry points.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import solution
from ._lib import PAGE_SIZE, TOPK

__all__ = ["shard_rows", "page_range", "split_row_topk", "gather_rows", "row_sharded_kernel"]


def shard_rows(seq_lens, world: int, rank: int) -> tuple[int, int]:
    """Contiguous rows [r0, r1) of `rank`, balanced by total tokens (each rank
    gets rows until its prefix of the token count passes its share)."""
    sl = np.asarray(seq_lens, dtype=np.int64).clip(min=0)
    rows = sl.shape[0]
    if world <= 1 or rows == 0:
        return 0, rows
    csum = np.concatenate([[0], np.cumsum(sl + 1)])  # +1 keeps empty rows spread
    total = csum[-1]
    bounds = [int(np.searchsorted(csum, total * g / world, side="left")) for g in range(world + 1)]
    bounds[0], bounds[-1] = 0, rows
    bounds = [min(max(b, 0), rows) for b in bounds]
    for g in range(1, world + 1):
        bounds[g] = max(bounds[g], bounds[g - 1])
    return bounds[rank], bounds[rank + 1]


def page_range(seq_len: int, world: int, rank: int) -> tuple[int, int]:
    """Pages [p0, p1) of a row of `seq_len` tokens that `rank` scores."""
    n_pages = (max(int(seq_len), 0) + PAGE_SIZE - 1) // PAGE_SIZE
    return n_pages * rank // world, n_pages * (rank + 1) // world


def _cuda_local_pairs(q_row, k_cache, weights_row, seq_len_local, bt_local, token_offset):
    dev = bt_local.device
    sc = torch.empty((1, TOPK), dtype=torch.float32, device=dev)
    tk = torch.empty((1, TOPK), dtype=torch.int32, device=dev)
    if bt_local.shape[1] == 0:  # this rank holds no page of the row
        sc.fill_(float("-inf"))
        tk.fill_(-1)
        return sc[0], tk[0]
    sl = torch.tensor([seq_len_local], dtype=torch.int32, device=dev)
    solution.run_pairs(q_row, k_cache, weights_row, sl, bt_local, token_offset, sc, tk)
    return sc[0], tk[0]


def _cuda_merge(scores, tokens, bt_row_full, seq_len, out):
    sl = torch.tensor([int(seq_len)], dtype=torch.int32, device=out.device)
    solution.merge_pairs(scores.contiguous(), tokens.contiguous(), bt_row_full.contiguous(), sl, out)


def split_row_topk(q_row, k_cache_local, weights_row, seq_len: int, bt_local_row, bt_full_row, out,
                   group=None, local_pairs=None, merge=None):
    """Top-2048 physical ids of ONE long row whose pages are spread over the
    ranks of `group` by page range (``page_range``).

    q_row [1, 64, 128], weights_row [1, 64]: the row's query and head weights
    (on every rank).  k_cache_local: this rank's K pool; bt_local_row
    [p1 - p0]: this rank's pages of the row, as ids into k_cache_local.
    bt_full_row [max_pages]: the row's full block table (global ids, used for
    the output).  out [2048] int32 receives the result on every rank.
    """
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    p0, p1 = page_range(seq_len, world, rank)
    local_len = max(0, min(int(seq_len), p1 * PAGE_SIZE) - p0 * PAGE_SIZE)
    bt_local = bt_local_row.reshape(1, -1)[:, : p1 - p0].contiguous()
    local_pairs = local_pairs or _cuda_local_pairs
    merge = merge or _cuda_merge
    sc, tk = local_pairs(q_row, k_cache_local, weights_row, local_len, bt_local, p0 * PAGE_SIZE)
    if world > 1:
        # one collective: the scores' fp32 bits and the tokens packed as
        # int32 [2, 2048] (16 KB per rank)
        packed = torch.stack([sc.contiguous().view(torch.int32), tk.contiguous()])
        bufs = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(bufs, packed, group=group)
        allp = torch.stack(bufs)                     # [world, 2, 2048]
        sc = allp[:, 0].reshape(-1).contiguous().view(torch.float32)
        tk = allp[:, 1].reshape(-1).contiguous()
    merge(sc, tk, bt_full_row, seq_len, out)
    return out


def row_sharded_kernel(q, k_cache, weights, seq_lens, block_table, topk_indices):
    """The indexer on this rank's rows (all arguments already hold only the
    rank's rows and pages).  Rows are independent: no collective."""
    solution.kernel(q, k_cache, weights, seq_lens, block_table, topk_indices)


def gather_rows(local_out: torch.Tensor, counts: list[int], group=None, buf: torch.Tensor | None = None) -> torch.Tensor:
    """All-gathers every rank's [rows_g, 2048] output into one [sum, 2048]
    tensor on every rank (rows_g given by `counts`).  One collective into a
    [world, max(counts), 2048] buffer (pass `buf` to reuse one across calls);
    the result is a view when every rank has the same row count."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return local_out
    world, m = len(counts), max(counts)
    if buf is None or tuple(buf.shape) != (world, m, TOPK) or buf.dtype != local_out.dtype:
        buf = torch.empty((world, m, TOPK), dtype=local_out.dtype, device=local_out.device)
    n = local_out.shape[0]
    if n == m:
        send = local_out.contiguous()
    else:
        send = torch.full((m, TOPK), -1, dtype=local_out.dtype, device=local_out.device)
        send[:n] = local_out
    if hasattr(dist, "all_gather_into_tensor") and dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(buf.view(world * m, TOPK), send, group=group)
    else:
        dist.all_gather(list(buf.unbind(0)), send, group=group)
    if all(c == m for c in counts):
        return buf.view(world * m, TOPK)
    return torch.cat([buf[g, :c] for g, c in enumerate(counts)])
