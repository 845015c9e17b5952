"""GPU test of dsai_run_noalloc, the entry point for callers that cannot
allocate device memory (a host that owns all device allocations and forbids
plugins to call cudaMalloc, a serving loop that bans allocation after
warm-up, a binding without a device allocator).  It keeps its workspace in a
16 MiB device array built into the library instead of taking one from the
caller.

Checked here through the C ABI: two calls in a row give the same top-2048 as
the ordinary entry point dsai_run (which gets its own workspace) — short rows
bit-exact, long rows the same set up to tokens whose logit ties the 2048th
largest (the tolerance the parity tests use; both paths compute identical
logits) — and the same answer as the CPU oracle under the parity rules of the
other GPU tests.  The array keeps the previous call's contents, so the second
call also checks that a call leaves it clean, and a third call with more rows
checks the newly used part of it.  After the calls the array's status word
(read through dsai_noalloc_read_status) must be clear.  This file is
collected last on purpose.
"""
import ctypes

import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import _lib
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOPK = 2048


def _args(g, out, logits=None, flags=0):
    a = _lib.DsaiArgs()
    a.q, a.k_cache, a.weights = g.q.data_ptr(), g.k_cache.data_ptr(), g.weights.data_ptr()
    a.seq_lens, a.block_table = g.seq_lens.data_ptr(), g.block_table.data_ptr()
    a.topk_indices = out.data_ptr()
    a.logits_out = logits.data_ptr() if logits is not None else None
    a.rows, a.max_pages, a.num_pages = g.rows, g.max_pages, g.num_pages
    a.flags = flags
    a.ev_after_score = None
    return a


def _expected(lib, g, stream):
    """Top-2048 and logits from the ordinary entry point, own workspace."""
    n = lib.dsai_workspace_size(g.rows, g.max_pages)
    ws = torch.empty(n, dtype=torch.uint8, device=DEV)
    assert lib.dsai_workspace_init(ws.data_ptr(), n, stream) == 0
    out = g.out()
    lg = torch.empty((g.rows, g.max_pages * 64), dtype=torch.float32, device=DEV)
    rc = lib.dsai_run(ctypes.byref(_args(g, out, lg, _lib.FLAG_SCORE_ALL_ROWS)), ws.data_ptr(), n, stream)
    assert rc == 0, lib.dsai_last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy(), lg.cpu().numpy()


def _same_topk(got, exp, logits, g):
    seq_lens = g.seq_lens.cpu().numpy()
    bt = g.block_table.cpu().numpy().astype(np.int64)
    for b, L in enumerate(seq_lens):
        if L <= TOPK:
            assert np.array_equal(got[b], exp[b]), f"row {b}: short row differs"
            continue
        assert len(set(got[b].tolist())) == TOPK, f"row {b}: duplicate ids"
        diff = set(got[b].tolist()) ^ set(exp[b].tolist())
        if diff:
            # only tokens whose logit ties the 2048th largest may be exchanged
            t = np.arange(L)
            token_of = dict(zip((bt[b, t // 64] * 64 + t % 64).tolist(), t.tolist()))
            row = logits[b, :L]
            kth = np.sort(row)[::-1][TOPK - 1]
            for pid in diff:
                assert row[token_of[pid]] == kth, f"row {b}: id {pid} differs outside the tie band"


def _noalloc_status(lib, stream):
    v = ctypes.c_int32(-1)
    assert lib.dsai_noalloc_read_status(stream, ctypes.byref(v)) == 0, lib.dsai_last_error()
    return int(v.value)


def _oracle_check(oracle_mod, inp, ids):
    """The no-alloc ids against the CPU oracle (parity rules of the GPU tests)."""
    d = inp.numpy()
    lg = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                           num_pages=d["num_pages"], nthreads=8)
    for b in range(inp.rows):
        oracle_mod.check_row(ids[b], lg[b], d["block_table"][b], int(d["seq_lens"][b]))


def test_noalloc_matches_run_on_two_calls_in_a_row(oracle_mod):
    lib = _lib.load_library()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    small_cpu = W.make_inputs([1500, 4096, 9001, 2049, 64, 20000], seed=41)
    small = small_cpu.to(DEV)
    exp, lg = _expected(lib, small, stream)
    for _ in range(2):
        out = small.out()
        rc = lib.dsai_run_noalloc(ctypes.byref(_args(small, out)), stream)
        assert rc == 0, lib.dsai_last_error()
        torch.cuda.synchronize()
        _same_topk(out.cpu().numpy(), exp, lg, small)
    _oracle_check(oracle_mod, small_cpu, out.cpu().numpy())
    assert _noalloc_status(lib, stream) == 0
    # more rows than before: part of the array that held logits now holds histograms
    big_cpu = W.config_inputs(1, rows=16, seed=42)
    big = big_cpu.to(DEV)
    exp2, lg2 = _expected(lib, big, stream)
    out = big.out()
    rc = lib.dsai_run_noalloc(ctypes.byref(_args(big, out)), stream)
    assert rc == 0, lib.dsai_last_error()
    torch.cuda.synchronize()
    _same_topk(out.cpu().numpy(), exp2, lg2, big)
    _oracle_check(oracle_mod, big_cpu, out.cpu().numpy())
    assert _noalloc_status(lib, stream) == 0


def test_noalloc_rejects_sizes_beyond_its_array():
    lib = _lib.load_library()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    a = _lib.DsaiArgs()
    a.rows, a.max_pages, a.num_pages = 256, 2048, 1  # ~134 MB of workspace
    assert lib.dsai_run_noalloc(ctypes.byref(a), stream) == -2
    assert b"static scratch" in lib.dsai_last_error()
