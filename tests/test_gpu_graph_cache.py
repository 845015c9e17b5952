"""GPU checks of the library's graph cache (``run(..., graph=True)``,
DSAI_FLAG_GRAPH): every call with fresh tensors (new pointers, as the
reference's benchmark harness passes them, solution/python/kernel.cu:1106-1110)
is replayed from one cached executable graph per launch plan and gives the
oracle's answer; new shapes and streams get plans of their own; a call made
while the caller's stream is capturing falls back to direct launches."""
import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import IndexerGraph, _lib, read_status, run
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _fresh(inp: W.Inputs) -> W.Inputs:
    """The same contents in newly allocated tensors."""
    return W.Inputs(inp.q.clone(), inp.k_cache.clone(), inp.weights.clone(), inp.seq_lens.clone(),
                    inp.block_table.clone(), rows_per_seq=inp.rows_per_seq)


def _check(oracle_mod, inp: W.Inputs, got: np.ndarray, lg=None, rows=None):
    d = inp.numpy()
    if lg is None:
        _, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    for b in (range(inp.rows) if rows is None else rows):
        L = int(min(max(d["seq_lens"][b], 0), inp.max_pages * 64))
        oracle_mod.check_row(got[b], lg[b], d["block_table"][b], L)


# (inputs, rows checked against the oracle: None = all)
CASES = {
    "scored": (lambda: W.make_inputs([1500, 4096, 9001, 2049, 30000, 0], max_pages=480, pool_pages=1500, seed=41), None),
    "short": (lambda: W.make_inputs([1, 63, 64, 65, 2048, 0, 700], max_pages=32, seed=42), None),
    "many_rows": (lambda: W.config_inputs(1, seed=43, rows=48), None),
    # more rows than one scoring launch takes (1024): three scoring launches and
    # the selection in one recorded plan
    "launch_chunks": (lambda: W.make_inputs(np.where(np.arange(2100) % 97 == 0, 3000, 2100).tolist(), seed=47),
                      [0, 1, 97, 1023, 1024, 1025, 2047, 2048, 2049, 2099]),
    # groups of four query rows sharing K pages (the grouped scorer)
    "groups": (lambda: W.config_inputs(4, seed=48, rows=16), None),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_graph_calls_with_fresh_tensors_match_oracle(oracle_mod, case):
    lib = _lib.load_library()
    make, check_rows = CASES[case]
    host = make()
    base = host.to(DEV)
    d = host.numpy()
    _, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    before = lib.dsai_graph_cache_entries()
    for it in range(4):
        g = _fresh(base)
        out = g.out()
        out.fill_(-7)
        run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, graph=True, rows_per_seq=g.rows_per_seq)
        torch.cuda.synchronize()
        _check(oracle_mod, host, out.cpu().numpy(), lg, check_rows)
        # one plan for all four calls: captured by the first, replayed after
        assert lib.dsai_graph_cache_entries() == before + 1
    assert read_status(DEV) == 0


def test_graph_plans_are_per_shape_and_stream(oracle_mod):
    lib = _lib.load_library()
    a = W.make_inputs([5000, 7000, 12000], max_pages=200, pool_pages=700, seed=44)
    b = W.make_inputs([5000, 7000, 12000, 3000], max_pages=200, pool_pages=700, seed=45)
    ga, gb = a.to(DEV), b.to(DEV)
    before = lib.dsai_graph_cache_entries()
    oa, ob = ga.out(), gb.out()
    run(ga.q, ga.k_cache, ga.weights, ga.seq_lens, ga.block_table, oa, graph=True)
    run(gb.q, gb.k_cache, gb.weights, gb.seq_lens, gb.block_table, ob, graph=True)
    torch.cuda.synchronize()
    assert lib.dsai_graph_cache_entries() == before + 2  # 3 and 4 rows: two plans
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):
        os_ = ga.out()
        run(ga.q, ga.k_cache, ga.weights, ga.seq_lens, ga.block_table, os_, graph=True)
    side.synchronize()
    assert lib.dsai_graph_cache_entries() == before + 3  # same shape, another stream
    _check(oracle_mod, a, oa.cpu().numpy())
    _check(oracle_mod, b, ob.cpu().numpy())
    _check(oracle_mod, a, os_.cpu().numpy())


def test_graph_flag_inside_a_capture_launches_directly(oracle_mod):
    """A call with the flag made while the caller captures its own graph is
    not replayed from the cache: its kernels go into the caller's graph."""
    lib = _lib.load_library()
    host = W.make_inputs([2500, 6000], max_pages=100, pool_pages=300, seed=46)
    g = host.to(DEV)
    out = g.out()
    ws = _lib.Workspace(DEV)
    side = torch.cuda.Stream(DEV)
    side.wait_stream(torch.cuda.current_stream(DEV))
    with torch.cuda.stream(side):  # sizes the workspace outside the capture
        run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, workspace=ws)
    torch.cuda.synchronize(DEV)
    before = lib.dsai_graph_cache_entries()
    cg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(cg, capture_error_mode="thread_local"):
        run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out, workspace=ws, graph=True)
    assert lib.dsai_graph_cache_entries() == before
    out.fill_(-7)
    cg.replay()
    torch.cuda.synchronize()
    _check(oracle_mod, host, out.cpu().numpy())
