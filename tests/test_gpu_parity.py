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


def test_concurrent_streams_have_separate_workspaces(oracle_mod):
    """Two different batches issued at once on two side streams, with no
    ordering between the streams: kernel() takes one default workspace per
    (device, stream), so neither call can overwrite the other's histograms,
    counters or logits.  Both results must match the oracle."""
    a = W.config_inputs(1, rows=6, seed=311)
    b = W.make_inputs([30000, 2500, 17000, 9000, 26000], seed=312)
    ga, gb = a.to(DEV), b.to(DEV)
    outs = [ga.out(), gb.out()]
    s1, s2 = torch.cuda.Stream(DEV), torch.cuda.Stream(DEV)
    cur = torch.cuda.current_stream(DEV)
    s1.wait_stream(cur)
    s2.wait_stream(cur)
    for _ in range(4):  # interleaved issue keeps both streams busy at once
        with torch.cuda.stream(s1):
            kernel(ga.q, ga.k_cache, ga.weights, ga.seq_lens, ga.block_table, outs[0])
        with torch.cuda.stream(s2):
            kernel(gb.q, gb.k_cache, gb.weights, gb.seq_lens, gb.block_table, outs[1])
    torch.cuda.synchronize()
    for s in (s1, s2):
        with torch.cuda.stream(s):
            assert read_status(DEV) == 0
    for inp, out in ((a, outs[0]), (b, outs[1])):
        ids = out.cpu().numpy()
        sel, lg, mag, d = oracle_rows(oracle_mod, inp)
        for i in range(inp.rows):
            oracle_mod.check_row(ids[i], lg[i], d["block_table"][i], int(d["seq_lens"][i]))
    # the two streams really did get different workspaces
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import _lib as L
    w1 = L.default_workspace(DEV, s1.cuda_stream)
    w2 = L.default_workspace(DEV, s2.cuda_stream)
    assert w1 is not w2 and w1.buf.data_ptr() != w2.buf.data_ptr()


def test_config1_full_size_all_rows(oracle_mod):
    """B=64, 4K-32K (the headline batch), production path: every row's ids
    and logits against the oracle, and every row an exact top-K of the
    GPU's own logits.  Tie-band differences are counted and printed."""
    inp = W.config_inputs(1)
    ids, glog, status = gpu_run(inp, score_all=False)
    assert status == 0
    sel, lg, mag, d = oracle_rows(oracle_mod, inp)
    worst = oracle_mod.check_logits(glog, lg, mag, d["seq_lens"])
    diffs = 0
    for b in range(inp.rows):
        r = oracle_mod.check_row(ids[b], lg[b], d["block_table"][b], int(d["seq_lens"][b]), gpu_logits=glog[b])
        diffs += r["diff"]
    print(f"config1: 64 rows checked, worst logit error {worst:.3g}, tie-band differences {diffs}")


def _pivot_bin_sizes(glog_dev, seq_lens):
    """Per row: keys in the 12-bit first-digit bin that holds the 2048th
    largest logit (the selection's pivot bin)."""
    sizes = []
    for b, L in enumerate(seq_lens.tolist()):
        if L <= TOPK:
            sizes.append(0)
            continue
        row = glog_dev[b, :L]
        u = row.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        key = torch.where(u >= 0x80000000, 0xFFFFFFFF - u, u | 0x80000000)
        bins = key >> 20
        kth = torch.topk(row, TOPK).values[-1:]
        ku = kth.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        kb = torch.where(ku >= 0x80000000, 0xFFFFFFFF - ku, ku | 0x80000000) >> 20
        sizes.append(int((bins == kb).sum().item()))
    return sizes


def _ids_in_subset(ids, bt_orig, bt_sub, L):
    """Rewrites physical ids of the full pool as ids of a compact subset pool."""
    t = np.arange(L)
    tok_of = dict(zip((bt_orig[t // 64].astype(np.int64) * 64 + t % 64).tolist(), t.tolist()))
    out = np.full_like(ids, -1)
    for j, p in enumerate(ids.tolist()):
        if p >= 0:
            tt = tok_of.get(int(p), -1)
            assert tt >= 0, "id not reachable through the block table"
            out[j] = int(bt_sub[tt // 64]) * 64 + tt % 64
    return out


def test_config2_full_batch_sampled_rows(oracle_mod):
    """Config 2 at full size (B=256, 64K-128K tokens, 3.3 GB pool built on
    the device): the whole batch through the production path, every row an
    exact top-K of its GPU logits, and sampled rows against the oracle: the
    longest row (four rounds of the one-CTA-per-row selection), the rows
    with the largest pivot bins (more than 2048 keys, where an earlier
    version fell back to a slow pass), and a few others."""
    inp = W.config_inputs(2, device=DEV)
    out = inp.out()
    glog = torch.full((inp.rows, inp.max_pages * 64), float("nan"), device=DEV)
    run(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out, logits_out=glog)
    torch.cuda.synchronize()
    assert read_status(DEV) == 0
    sl = inp.seq_lens.cpu().numpy()
    sizes = _pivot_bin_sizes(glog, inp.seq_lens.cpu())
    ids_all = out.cpu().numpy()
    bt_all = inp.block_table.cpu().numpy()
    # every row: an exact top-K of the GPU's own logits, distinct reachable ids
    for b in range(inp.rows):
        L = int(sl[b])
        row = glog[b, :L]
        t = torch.arange(L, device=DEV)
        phys = inp.block_table[b, t // 64].long() * 64 + t % 64
        inv = torch.full((int(phys.max()) + 1,), -1, dtype=torch.long, device=DEV)
        inv[phys] = t
        ids = out[b].long()
        assert bool((ids >= 0).all()) and bool((ids <= phys.max()).all()), f"row {b}"
        toks = inv[ids]
        assert bool((toks >= 0).all()) and int(torch.unique(toks).numel()) == TOPK, f"row {b}"
        m = torch.zeros(L, dtype=torch.bool, device=DEV)
        m[toks] = True
        assert bool(row[m].min() >= row[~m].max()), f"row {b}"
    order = np.argsort(sizes)[::-1]
    rows = sorted({int(np.argmax(sl))} | set(int(r) for r in order[:4]) | {0, 97, 255})
    sub = inp.subset(rows)
    d = sub.numpy()
    lg, mag = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                                num_pages=d["num_pages"], nthreads=8, with_mag=True)
    g_sub = glog[rows].cpu().numpy()
    worst = oracle_mod.check_logits(g_sub, lg, mag, d["seq_lens"])
    diffs = 0
    for i, b in enumerate(rows):
        L = int(sl[b])
        mapped = _ids_in_subset(ids_all[b], bt_all[b], d["block_table"][i], L)
        r = oracle_mod.check_row(mapped, lg[i], d["block_table"][i], L, gpu_logits=g_sub[i])
        diffs += r["diff"]
    print(f"config2: rows {rows} (L max {int(sl.max())}, pivot bins {[sizes[r] for r in rows]}) "
          f"worst logit error {worst:.3g}, tie-band differences {diffs}")


def test_row_chunking_over_launch_limit(oracle_mod):
    """More rows than one scoring launch handles (1024): five launches."""
    rows = 4100
    lens = np.full(rows, 2100)
    lens[::97] = 3000
    inp = W.make_inputs(lens, seed=27)
    ids, glog, status = gpu_run(inp, score_all=False)
    assert status == 0
    check(oracle_mod, inp, ids, glog, rows=[0, 1, 1023, 1024, 2048, 4095, 4096, 4099])
