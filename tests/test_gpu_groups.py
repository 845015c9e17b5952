"""GPU parity of the group scorer (rows_per_seq = 2..4: consecutive rows that
are query tokens of one sequence read its K pages once).

Its logits must be bit-identical to those of the per-row scorer (same
arithmetic in the same order), which the oracle pins within the north-star
tolerances (rtol 1e-2 on logits, identical index sets outside the tie band,
rows with seq_len <= 2048 and -1 padding bit-exact).
"""
import ctypes

import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import IndexerGraph, _lib, read_status, run
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200.solution import _args

from test_gpu_parity import check

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def gpu_run(g, rows_per_seq, score_all=True):
    out = g.out()
    lg = torch.full((g.rows, g.max_pages * 64), float("nan"), device=DEV)
    run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, logits_out=lg,
        score_all_rows=score_all, rows_per_seq=rows_per_seq)
    torch.cuda.synchronize()
    return out.cpu().numpy(), lg.cpu().numpy(), read_status(DEV)


def same_logits(a, b, lens):
    for r, L in enumerate(lens):
        L = max(0, int(L))
        assert np.array_equal(a[r, :L].view(np.uint32), b[r, :L].view(np.uint32)), f"row {r}"


def same_ids(a, b, lens):
    for r, L in enumerate(lens):
        if L <= 2048:
            assert np.array_equal(a[r], b[r]), f"row {r}"
        else:
            assert set(a[r].tolist()) == set(b[r].tolist()), f"row {r}"


@pytest.mark.parametrize("R", [2, 3, 4])
def test_groups_match_rows_and_oracle(oracle_mod, R):
    """Causal group lengths (L-R+1 .. L), groups mixing rows on both sides of
    2048, a group of short rows only (not scored), an empty row."""
    rng = np.random.default_rng(40 + R)
    lens = []
    for base in [9000, 2049, 300, 20000, 4100]:
        lens += [base - (R - 1) + i for i in range(R)]
    lens += rng.integers(5000, 15000, R * 3).tolist()
    lens[-1] = 0
    inp = W.make_inputs([max(1, L) for L in lens], seed=50 + R, share_rows=R)
    inp.seq_lens = torch.tensor(lens, dtype=torch.int32)
    g = inp.to(DEV)
    ids_g, lg_g, st_g = gpu_run(g, R)
    ids_r, lg_r, st_r = gpu_run(g, 1)
    assert st_g == 0 and st_r == 0
    same_logits(lg_g, lg_r, lens)
    same_ids(ids_g, ids_r, lens)
    check(oracle_mod, inp, ids_g, lg_g)
    # the production path (short rows not scored) gives the same ids
    ids_p, _, _ = gpu_run(g, R, score_all=False)
    same_ids(ids_p, ids_g, lens)


def test_config4_groups(oracle_mod):
    inp = W.config_inputs(4, rows=16)
    assert inp.rows_per_seq == 4
    g = inp.to(DEV)
    ids_g, lg_g, st = gpu_run(g, 4, score_all=False)
    ids_r, lg_r, _ = gpu_run(g, 1, score_all=False)
    assert st == 0
    lens = inp.seq_lens.numpy()
    same_logits(lg_g, lg_r, lens)
    same_ids(ids_g, ids_r, lens)
    check(oracle_mod, inp, ids_g, lg_g, rows=[0, 3, 5, 10, 15])


def test_group_reads_longest_rows_block_table(oracle_mod):
    """Only the pages a row reaches must agree inside a group: entries past a
    row's own length are garbage, and the longest row is not the first."""
    lens = [7000, 9000, 8000, 3000]
    inp = W.make_inputs(lens, seed=61, share_rows=4)
    bt = inp.block_table.clone()
    for r, L in enumerate(lens):
        bt[r, (L + 63) // 64:] = -99
    inp.block_table = bt
    g = inp.to(DEV)
    ids_g, lg_g, st = gpu_run(g, 4)
    assert st == 0
    check(oracle_mod, inp, ids_g, lg_g)


def test_full_config4_all_rows(oracle_mod):
    """All 128 rows of config 4: the group path equals the per-row path, bit
    for bit on logits and as sets on ids, and every row matches the oracle
    (logits and ids; tie-band differences counted)."""
    inp = W.config_inputs(4)
    g = inp.to(DEV)
    ids_g, lg_g, st = gpu_run(g, 4, score_all=False)
    ids_r, lg_r, _ = gpu_run(g, 1, score_all=False)
    assert st == 0
    lens = inp.seq_lens.numpy()
    same_logits(lg_g, lg_r, lens)
    same_ids(ids_g, ids_r, lens)
    diffs = check(oracle_mod, inp, ids_g, lg_g)
    print(f"config4: 128 rows checked, tie-band differences {diffs}")


def test_groups_over_launch_limit():
    """1032 rows in groups of 4: two scoring launches, the second starting
    at row 1024."""
    rows = 1032
    lens = np.full(rows, 2100)
    lens[1::7] = 2600
    inp = W.make_inputs(lens, seed=62, share_rows=4)
    g = inp.to(DEV)
    ids_g, lg_g, st = gpu_run(g, 4, score_all=False)
    ids_r, lg_r, _ = gpu_run(g, 1, score_all=False)
    assert st == 0
    same_logits(lg_g, lg_r, lens)
    same_ids(ids_g, ids_r, lens)


@pytest.mark.parametrize("chunk,last_len", [(32, 12000), (32, 2061)])
def test_prefill_chunk(oracle_mod, chunk, last_len):
    """A prefill chunk (causal rows of one sequence over one block table) in
    groups of 4; the second chunk crosses 2048, so its first groups mix rows
    that are all selected with scored rows."""
    inp = W.prefill_inputs(chunk, last_len, seed=64)
    g = inp.to(DEV)
    lens = inp.seq_lens.numpy()
    ids_g, lg_g, st = gpu_run(g, 4)
    ids_r, lg_r, _ = gpu_run(g, 1)
    assert st == 0
    same_logits(lg_g, lg_r, lens)
    same_ids(ids_g, ids_r, lens)
    check(oracle_mod, inp, ids_g, lg_g, rows=[0, 5, 17, chunk - 1])


def test_group_arguments_rejected():
    inp = W.make_inputs([3000, 3000, 3000], seed=63).to(DEV)
    out = inp.out()
    with pytest.raises(RuntimeError):
        run(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out, rows_per_seq=2)
    with pytest.raises(RuntimeError):
        run(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out, rows_per_seq=5)
    # the C ABI checks the same on its own
    lib = _lib.load_library()
    ws = _lib.Workspace(DEV)
    stream = torch.cuda.current_stream(DEV).cuda_stream
    ws_ptr, ws_bytes = ws.get(inp.rows, inp.max_pages, stream)
    for rps in (2, 5, -1):
        a = _args(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out, None, 0, rps)
        assert lib.dsai_run(ctypes.byref(a), ws_ptr, ws_bytes, stream) == _lib.E_INVALID
    torch.cuda.synchronize()


def test_group_graph_replay():
    inp = W.config_inputs(4, rows=8).to(DEV)
    out = inp.out()
    graph = IndexerGraph(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out, rows_per_seq=4)
    out.fill_(-7)
    graph.replay()
    ref = inp.out()
    run(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, ref)
    torch.cuda.synchronize()
    same_ids(out.cpu().numpy(), ref.cpu().numpy(), inp.seq_lens.cpu().numpy())
