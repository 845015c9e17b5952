"""The indexer as a plain PyTorch CPU computation — TEST / BASELINE
INFRASTRUCTURE ONLY (bench.py's CPU baseline leg and reference arm, tests).

This is the torch formulation of the reference's operator that its
definition describes (solution/cuda/kernel.cu:4-21, solution/python/
kernel.cu:5-9), run on the host cores with torch's own thread pool:

  per row, per chunk of its pages (block_table[b, t/64]):
    K  = e4m3 bytes of the chunk's pages -> fp32            [n*64, 128]
    S  = K @ q[b]^T                                          [n*64, 64]   (fp32 GEMM)
    lg = (ReLU(S) @ weights[b]) * scale[page, slot]          [n*64]
  top-2048 of lg[0:L] (torch.topk), then physical ids bt[t/64]*64 + t%64
  (solution/python/kernel.cu:1021-1027); rows with L <= 2048 give tokens
  0..L-1 in order and -1 padding (kernel.cu:897-905, :1079-1097).

fp32 throughout (the GEMM accumulates in fp32, as the reference's tcgen05
MMA does), so near-ties may order differently from the exact C oracle;
tests/test_torch_path.py checks it against that oracle within the
north-star tolerances.
"""
from __future__ import annotations

import numpy as np
import torch

TOPK = 2048
PAGE = 64
PAGE_BYTES = 8448
SCALE_OFF = 8192


def row_logits(q_row: torch.Tensor, w_row: torch.Tensor, k_pages: torch.Tensor, pages: torch.Tensor,
               L: int, chunk_pages: int = 512) -> torch.Tensor:
    """fp32 logits of one row over tokens [0, L): q_row [64, 128] fp32,
    w_row [64] fp32, k_pages [num_pages, 8448] uint8, pages [>= ceil(L/64)]."""
    npg = (L + PAGE - 1) // PAGE
    out = torch.empty(npg * PAGE, dtype=torch.float32)
    qt = q_row.t().contiguous()                                        # [128, 64]
    for c0 in range(0, npg, chunk_pages):
        pg = pages[c0:min(npg, c0 + chunk_pages)].long()
        blk = k_pages.index_select(0, pg)                                  # [n, 8448] u8
        k = blk[:, :SCALE_OFF].contiguous().view(torch.float8_e4m3fn).to(torch.float32).view(-1, 128)
        sc = blk[:, SCALE_OFF:].contiguous().view(torch.float32).reshape(-1)
        s = torch.mm(k, qt)                                                # [n*64, 64]
        out[c0 * PAGE:c0 * PAGE + s.shape[0]] = torch.mv(torch.relu_(s), w_row) * sc
    return out[:L]


def indexer(q_u8: np.ndarray, k_cache_u8: np.ndarray, weights: np.ndarray, seq_lens: np.ndarray,
            block_table: np.ndarray, rows=None, return_logits: bool = False):
    """Top-2048 physical ids [len(rows), 2048] int32 (-1 padded) of the
    given rows (default: all); with return_logits also the per-row fp32
    logits (list of arrays)."""
    q = torch.from_numpy(np.ascontiguousarray(q_u8)).view(torch.float8_e4m3fn).to(torch.float32)
    q = q.view(-1, 64, 128)
    kp = torch.from_numpy(np.ascontiguousarray(k_cache_u8)).view(-1, PAGE_BYTES)
    w = torch.from_numpy(np.ascontiguousarray(weights, dtype=np.float32)).view(-1, 64)
    bt = torch.from_numpy(np.ascontiguousarray(block_table, dtype=np.int32))
    sl = np.asarray(seq_lens).astype(np.int64)
    rows = range(q.shape[0]) if rows is None else rows
    outs, lgs = [], []
    for b in rows:
        L = int(min(max(sl[b], 0), bt.shape[1] * PAGE))
        ids = torch.full((TOPK,), -1, dtype=torch.int64)
        if L <= TOPK:
            t = torch.arange(L)
            ids[:L] = bt[b, t // PAGE].long() * PAGE + t % PAGE
            lgs.append(None)
        else:
            lg = row_logits(q[b], w[b], kp, bt[b], L)
            top = torch.topk(lg, TOPK, sorted=False).indices
            ids[:] = bt[b, top // PAGE].long() * PAGE + top % PAGE
            lgs.append(lg.numpy())
        outs.append(ids.to(torch.int32))
    ids = torch.stack(outs).numpy() if outs else np.zeros((0, TOPK), np.int32)
    return (ids, lgs) if return_logits else ids
