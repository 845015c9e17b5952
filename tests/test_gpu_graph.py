"""GPU checks of IndexerGraph: a captured indexer call replayed on the same
tensors gives the eager result, also after the tensors' contents are
replaced in place (new queries, weights, lengths and K pages)."""
import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import IndexerGraph, kernel
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _check(oracle_mod, inp, got):
    d = inp.numpy()
    exp, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    for b in range(inp.rows):
        L = int(min(max(d["seq_lens"][b], 0), inp.max_pages * 64))
        oracle_mod.check_row(got[b], lg[b], d["block_table"][b], L)  # raises on a mismatch


def test_graph_replays_match_eager_and_follow_new_contents(oracle_mod):
    a = W.make_inputs([1500, 4096, 9001, 2049], max_pages=160, pool_pages=700, seed=31)
    b = W.make_inputs([3000, 10240, 64, 7000], max_pages=160, pool_pages=700, seed=32)
    g = a.to(DEV)
    out = g.out()
    graph = IndexerGraph(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, out)
    for _ in range(2):
        out.fill_(-7)
        graph.replay()
        torch.cuda.synchronize()
        _check(oracle_mod, a, out.cpu().numpy())
    # new contents, same tensors
    nb = b.to(DEV)
    for dst, src in ((g.q, nb.q), (g.k_cache, nb.k_cache), (g.weights, nb.weights),
                     (g.seq_lens, nb.seq_lens), (g.block_table, nb.block_table)):
        dst.copy_(src)
    graph.replay()
    torch.cuda.synchronize()
    _check(oracle_mod, b, out.cpu().numpy())
    eager = nb.out()
    kernel(nb.q, nb.k_cache, nb.weights, nb.seq_lens, nb.block_table, eager)
    torch.cuda.synchronize()
    short = np.asarray(b.seq_lens.cpu()) <= 2048
    assert np.array_equal(out.cpu().numpy()[short], eager.cpu().numpy()[short])
