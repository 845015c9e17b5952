"""GPU parity of the CUDA path against the CPU oracle, through the drop-in
entry point and the C ABI it calls.

Tolerances: logits within rtol 1e-2 of the oracle
(plus 1e-4 of the head-sum magnitude, which bounds cancellation); index sets
identical outside the tie band rtol*|s_2048|, differences inside it counted;
rows with seq_len <= 2048 and -1 padding bit-exact.  Every long row is also
checked to be an exact top-K of the GPU's own logits.
"""
import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import _lib, kernel, read_status, run
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOPK = 2048


def gpu_run(inp, score_all=True):
    g = inp.to(DEV)
    out = g.out()
    lg = torch.full((g.rows, g.max_pages * 64), float("nan"), device=DEV)
    run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, logits_out=lg, score_all_rows=score_all)
    torch.cuda.synchronize()
    status = read_status(DEV)
    return out.cpu().numpy(), lg.cpu().numpy(), status


def oracle_rows(oracle_mod, inp, rows=None):
    d = inp.numpy()
    sel = np.arange(inp.rows) if rows is None else np.asarray(rows)
    lg, mag = oracle_mod.logits(d["q"][sel], d["k_cache"], d["weights"][sel], d["seq_lens"][sel],
                                d["block_table"][sel], num_pages=d["num_pages"], nthreads=8, with_mag=True)
    return sel, lg, mag, d


def check(oracle_mod, inp, ids, glog, rows=None):
    sel, lg, mag, d = oracle_rows(oracle_mod, inp, rows)
    oracle_mod.check_logits(glog[sel], lg, mag, d["seq_lens"][sel])
    diffs = 0
    for i, b in enumerate(sel):
        L = int(min(max(d["seq_lens"][b], 0), inp.max_pages * 64))
        r = oracle_mod.check_row(ids[b], lg[i], d["block_table"][b], L, gpu_logits=glog[b])
        diffs += r["diff"]
    return diffs


def test_config0_full(oracle_mod):
    inp = W.config_inputs(0)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)
    # the plain drop-in gives the same ids (short row bit-exact, long row same set)
    g = inp.to(DEV)
    out = g.out()
    assert kernel(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out) is None
    o = out.cpu().numpy()
    assert np.array_equal(o[0], ids[0])
    assert set(o[1].tolist()) == set(ids[1].tolist())


def test_logits_match_published_reference_golden(oracle_mod):
    """GPU logits (every row scored) against the golden logits of DeepGEMM's
    published paged FP8 MQA logits reference (tests/golden/)."""
    import sys
    from pathlib import Path
    gdir = Path(__file__).resolve().parent / "golden"
    sys.path.insert(0, str(gdir))
    import make_indexer_logits_golden as G
    z = np.load(gdir / "indexer_logits_golden.npz")
    inp = G.inputs()
    assert G.digest(inp) == str(z["sha256"])
    ids, glog, status = gpu_run(inp)
    assert status == 0
    d = inp.numpy()
    _, mag = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                               num_pages=d["num_pages"], nthreads=8, with_mag=True)
    g = np.concatenate([glog[b, :L] for b, L in enumerate(G.LENS)])
    m = np.concatenate([mag[b, :L] for b, L in enumerate(G.LENS)])
    assert np.all(np.abs(g - z["logits"]) <= 1e-4 * (np.abs(z["logits"]) + m))
    check(oracle_mod, inp, ids, glog)


def test_config1_rows(oracle_mod):
    inp = W.config_inputs(1, rows=6)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)


def test_edge_lengths_mixed_batch(oracle_mod):
    lens = [0, 1, 63, 64, 65, 127, 128, 129, 2047, 2048, 2049, 2050, 4097, 6000]
    inp = W.make_inputs([max(1, L) for L in lens], max_pages=100, seed=21)
    inp.seq_lens = torch.tensor(lens, dtype=torch.int32)
    # entries past each row's last page are never read: fill them with garbage
    bt = inp.block_table.clone()
    for b, L in enumerate(lens):
        bt[b, (L + 63) // 64:] = -123456
    inp.block_table = bt
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)
    # without debug scoring (the production path) short rows are identical
    ids2, _, _ = gpu_run(inp, score_all=False)
    assert np.array_equal(ids2[:10], ids[:10])
    for b in range(10, len(lens)):
        assert set(ids2[b].tolist()) == set(ids[b].tolist())


def test_all_short_rows_fast_path(oracle_mod):
    inp = W.make_inputs([5, 2048, 700, 1], max_pages=32, seed=22)
    g = inp.to(DEV)
    out = g.out()
    kernel(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out)
    d = inp.numpy()
    exp = oracle_mod.topk(np.zeros((4, 32 * 64), np.float32), d["seq_lens"], d["block_table"])
    assert np.array_equal(out.cpu().numpy(), exp)


def test_long_rows_beyond_smem_cache(oracle_mod):
    """Long rows: several selection chunks and a large pivot bin."""
    inp = W.make_inputs([45000, 70001], seed=23)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)


def test_multi_query_shared_block_table(oracle_mod):
    inp = W.config_inputs(4, rows=8)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)


def test_ties_all_equal_logits(oracle_mod):
    """q = 0 makes every logit 0: any 2048 distinct reachable ids are right."""
    inp = W.make_inputs([5000, 3000], seed=24)
    inp.q = torch.zeros_like(inp.q)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)
    assert np.all(glog[0, :5000] == 0)


def test_ties_overflow_candidate_lists(oracle_mod):
    """One long row of equal logits: every CTA of the row's cluster finds
    more pivot-bin keys than its list holds, so the selection falls back to
    refining over the row in global memory."""
    inp = W.make_inputs([40000], seed=27)
    inp.q = torch.zeros_like(inp.q)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)
    assert np.all(glog[0, :40000] == 0)


def test_one_cta_per_row_paths(oracle_mod):
    """A batch large enough for one selection CTA per row, mixing the
    refinement paths: an all-equal row longer than the pivot list (refine
    over the row), an all-equal row that fits it (third digit over the list),
    64-token groups of equal logits, rows at the 2048 boundary, and ordinary
    rows (second digit, then one warp ranks the last keys)."""
    rng = np.random.default_rng(28)
    lens = [20000, 5000, 30000, 2048, 2049] + rng.integers(3000, 12000, 35).tolist()
    inp = W.make_inputs(lens, seed=28)
    inp.q[0].zero_()
    inp.q[1].zero_()
    bt2 = inp.block_table[2, : (30000 + 63) // 64].long()
    flat = inp.k_cache.view(-1, 8448)
    flat[bt2, 128:8192] = flat[bt2, 0:128].repeat(1, 63)
    flat[bt2, 8192 + 4:8448] = flat[bt2, 8192:8196].repeat(1, 63)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)
    assert np.all(glog[0, :20000] == 0) and np.all(glog[1, :5000] == 0)


def test_many_ties_in_pivot_bucket(oracle_mod):
    """Quantised logits with heavy ties around the boundary (the pivot bin
    overflows the candidate list and the refinement re-reads the row)."""
    inp = W.make_inputs([30000], seed=25)
    # all K tokens identical per page -> 64-token groups of equal logits
    flat = inp.k_cache.view(-1, 8448)
    flat[:, 128:8192] = flat[:, 0:128].repeat(1, 63)
    flat[:, 8192 + 4:8448] = flat[:, 8192:8196].repeat(1, 63)
    ids, glog, status = gpu_run(inp)
    assert status == 0
    check(oracle_mod, inp, ids, glog)


def test_invalid_inputs_flagged_not_faulting(oracle_mod):
    inp = W.make_inputs([3000, 3000, 100], seed=26)
    bt = inp.block_table.clone()
    bt[1, 5] = inp.num_pages + 1000  # page out of range -> zero page, flagged
    inp.block_table = bt
    sl = inp.seq_lens.clone()
    sl[2] = 1 << 30               # clamped to max_pages*64, flagged
    inp.seq_lens = sl
    ids, glog, status = gpu_run(inp)
    assert status & _lib.STATUS_BAD_PAGE
    assert status & _lib.STATUS_SEQLEN_CLAMPED
    assert not status & _lib.STATUS_WAIT_TIMEOUT
    assert np.all(glog[1, 5 * 64:6 * 64] == 0.0)
    check(oracle_mod, inp, ids, glog, rows=[0, 1])
    assert read_status(DEV) == 0  # reading clears


def test_repeatable_and_dps():
    inp = W.config_inputs(1, rows=4).to(DEV)
    outs = []
    for _ in range(3):
        out = inp.out()
        kernel(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out)
        outs.append(out.cpu().numpy())
    for o in outs[1:]:
        for b in range(4):
            assert set(o[b].tolist()) == set(outs[0][b].tolist())


def test_streams_are_honoured():
    inp = W.config_inputs(1, rows=4).to(DEV)
    s = torch.cuda.Stream(DEV)
    ref = inp.out()
    kernel(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, ref)
    out = inp.out()
    with torch.cuda.stream(s):
        kernel(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out)
    s.synchronize()
    for b in range(4):
        assert set(out[b].tolist()) == set(ref[b].tolist())


def test_config1_full_size_properties(oracle_mod):
    """B=64, 4K-32K: every row an exact top-K of its GPU logits, logits of a
    few sampled rows against the oracle."""
    inp = W.config_inputs(1)
    ids, glog, status = gpu_run(inp, score_all=False)
    assert status == 0
    check(oracle_mod, inp, ids, glog, rows=[0, 31, 63])
    d = inp.numpy()
    for b in range(inp.rows):
        L = int(d["seq_lens"][b])
        phys = oracle_mod.physical_ids(d["block_table"][b], L)
        tok_of = dict(zip(phys.tolist(), range(L)))
        toks = np.array([tok_of[int(p)] for p in ids[b]])
        assert len(set(toks.tolist())) == TOPK
        sel = np.zeros(L, bool)
        sel[toks] = True
        assert glog[b, :L][sel].min() >= glog[b, :L][~sel].max()


def test_row_chunking_over_launch_limit(oracle_mod):
    """More rows than one scoring launch handles (1024): five launches."""
    rows = 4100
    lens = np.full(rows, 2100)
    lens[::97] = 3000
    inp = W.make_inputs(lens, seed=27)
    ids, glog, status = gpu_run(inp, score_all=False)
    assert status == 0
    check(oracle_mod, inp, ids, glog, rows=[0, 1, 1023, 1024, 2048, 4095, 4096, 4099])
