"""GPU parity of the page-range split of one long row (the multi-GPU path of
a single long request), emulated on one GPU: each "rank" scores its page
range with dsai_run_pairs, the pairs are concatenated as the all-gather would,
and dsai_merge_pairs selects the row's top-2048.  Compared with the direct
indexer and with the CPU oracle."""
import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import distributed as D
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import kernel, merge_pairs, run, run_pairs
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TOPK = 2048


def emulated_split(g, world):
    L = int(g.seq_lens[0])
    scs, tks = [], []
    for r in range(world):
        p0, p1 = D.page_range(L, world, r)
        sc = torch.empty((1, TOPK), dtype=torch.float32, device=DEV)
        tk = torch.empty((1, TOPK), dtype=torch.int32, device=DEV)
        if p1 == p0:
            sc.fill_(float("-inf")); tk.fill_(-1)
        else:
            local_len = min(L, p1 * 64) - p0 * 64
            sl = torch.tensor([local_len], dtype=torch.int32, device=DEV)
            run_pairs(g.q, g.k_cache, g.weights, sl, g.block_table[:, p0:p1].contiguous(), p0 * 64, sc, tk)
        scs.append(sc[0]); tks.append(tk[0])
    out = torch.empty(TOPK, dtype=torch.int32, device=DEV)
    merge_pairs(torch.cat(scs), torch.cat(tks), g.block_table[0].contiguous(),
                g.seq_lens[:1].contiguous(), out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("world", [1, 2, 4, 8, 16])
def test_config3_split_matches_direct_and_oracle(oracle_mod, world):
    inp = W.config_inputs(3)          # B=1, L=131072, 16 planted tokens
    g = inp.to(DEV)
    merged = emulated_split(g, world)
    direct = g.out()
    lg = torch.empty((1, g.max_pages * 64), dtype=torch.float32, device=DEV)
    run(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, direct, logits_out=lg)
    torch.cuda.synchronize()
    d = inp.numpy()
    ora, mag = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                                 nthreads=8, with_mag=True)
    oracle_mod.check_logits(lg.cpu().numpy(), ora, mag, d["seq_lens"])
    L = int(d["seq_lens"][0])
    oracle_mod.check_row(merged, ora[0], d["block_table"][0], L, gpu_logits=lg.cpu().numpy()[0])
    oracle_mod.check_row(direct.cpu().numpy()[0], ora[0], d["block_table"][0], L)
    planted = oracle_mod.physical_ids(d["block_table"][0], L)[inp.planted[0]]
    assert set(planted.tolist()) <= set(merged.tolist())


@pytest.mark.parametrize("L", [1500, 2048, 2049, 5000])
def test_split_short_and_boundary_rows(oracle_mod, L):
    inp = W.make_inputs([L], seed=L)
    g = inp.to(DEV)
    merged = emulated_split(g, 3)
    d = inp.numpy()
    ora = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    oracle_mod.check_row(merged, ora[0], d["block_table"][0], L)


def test_pairs_short_rows_and_offsets(oracle_mod):
    inp = W.make_inputs([700, 3000], seed=5)
    g = inp.to(DEV)
    sc = torch.empty((2, TOPK), dtype=torch.float32, device=DEV)
    tk = torch.empty((2, TOPK), dtype=torch.int32, device=DEV)
    run_pairs(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, 1000, sc, tk)
    torch.cuda.synchronize()
    tk = tk.cpu().numpy(); sc = sc.cpu().numpy()
    assert np.array_equal(tk[0, :700], np.arange(700) + 1000) and np.all(tk[0, 700:] == -1)
    assert np.all(np.isneginf(sc[0, 700:]))
    d = inp.numpy()
    ora = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    osc, otk = oracle_mod.pairs(ora, d["seq_lens"], 1000)
    assert set(tk[1].tolist()) == set(otk[1].tolist())


def test_merge_list_no_longer_than_topk():
    """A candidate list of at most 2048 entries (one rank's pairs): every real
    entry is selected, padding (-1) and tokens past the row are not."""
    inp = W.make_inputs([6000], seed=31)
    g = inp.to(DEV)
    gen = torch.Generator().manual_seed(31)
    tokens = torch.randperm(6000, generator=gen)[:2048].to(torch.int32)
    tokens[::7] = -1          # padding
    tokens[3::11] = 7000      # past the row's end
    scores = torch.randn(2048, generator=gen)
    out = torch.empty(TOPK, dtype=torch.int32, device=DEV)
    merge_pairs(scores.to(DEV), tokens.to(DEV), g.block_table[0].contiguous(), g.seq_lens[:1].contiguous(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    bt = inp.block_table[0].numpy()
    real = tokens.numpy()
    real = real[(real >= 0) & (real < 6000)]
    expect = bt[real // 64] * 64 + real % 64
    n = len(expect)
    assert np.array_equal(np.sort(got[:n]), np.sort(expect))
    assert np.all(got[n:] == -1)
