"""CPU tests of the oracle (the parity checker): format decoding, known-answer
cases computed by hand, agreement of the two restatements (C and numpy),
the short-row contract, malformed-input conventions, the merge semantics
of a split row, and the parity checker itself (with planted mistakes)."""
import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

TOPK = 2048


def _inputs_np(inp):
    d = inp.numpy()
    return d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"]


def test_e4m3_decode_matches_torch_and_numpy(oracle_mod):
    t = oracle_mod.e4m3_table()
    n = oracle_mod._e4m3_numpy()
    tt = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).to(torch.float64).numpy()
    assert np.array_equal(np.isnan(t), np.isnan(tt))
    finite = ~np.isnan(t)
    assert np.array_equal(t[finite], tt[finite])
    assert np.array_equal(t[finite], n[finite])
    assert np.nanmax(t) == 448.0 and np.isnan(t[0x7F]) and np.isnan(t[0xFF])
    assert t[0x01] == 2.0 ** -9  # smallest subnormal


def test_ordered_key_is_monotone(oracle_mod):
    L = oracle_mod.lib()
    vals = np.array([-np.inf, -3.5, -1e-30, -0.0, 0.0, 1e-30, 2.0, np.inf], dtype=np.float32)
    keys = [L.dsai_oracle_key(float(v)) for v in vals]
    assert keys == sorted(keys) and len(set(keys)) == len(keys)


def test_page_pack_roundtrip_and_quantisation():
    g = torch.Generator().manual_seed(3)
    k = torch.randn(3 * 64, 128, generator=g)
    kq, sc = W.quantize_tokens(k)
    assert torch.allclose(sc, k.abs().amax(-1) / 448.0)
    assert kq.to(torch.float32).abs().amax(-1).eq(448.0).all()
    packed = W.pack_pages(kq, sc)
    assert packed.shape == (3, 64, 1, 132) and packed.dtype == torch.uint8
    kq2, sc2 = W.unpack_pages(packed)
    assert torch.equal(kq2.view(torch.uint8).reshape(-1, 128), kq.view(torch.uint8))
    assert torch.equal(sc2.reshape(-1), sc)
    # layout: token s of page p at byte p*8448 + s*128, its scale at p*8448 + 8192 + 4s
    flat = packed.reshape(-1).numpy()
    p, s = 2, 37
    tok = p * 64 + s
    assert np.array_equal(flat[p * 8448 + s * 128: p * 8448 + s * 128 + 128], kq[tok].view(torch.uint8).numpy())
    assert flat[p * 8448 + 8192 + 4 * s: p * 8448 + 8192 + 4 * s + 4].view(np.float32)[0] == sc[tok].item()


def _one_hot_case(weights_sign=1.0):
    """q[h] = e_h (1.0 at d = h), so S_h = k[h]; K values from a small exact
    set; logit = scale * sum_{h<64} max(k[h], 0) * w[h]."""
    vals = np.array([-2.0, -1.0, -0.5, 0.0, 0.5, 1.0, 2.0, 4.0], dtype=np.float32)
    rng = np.random.RandomState(11)
    L = 40
    k = vals[rng.randint(0, len(vals), size=(64, 128))].astype(np.float32)
    q = np.zeros((1, 64, 128), dtype=np.float32)
    q[0, np.arange(64), np.arange(64)] = 1.0
    w = (weights_sign * (np.arange(64, dtype=np.float32) + 1) / 64.0)[None, :].astype(np.float32)
    scale = (np.arange(64, dtype=np.float32) + 1) * 0.25
    kq = torch.from_numpy(k).to(torch.float8_e4m3fn)
    assert np.array_equal(kq.to(torch.float32).numpy(), k)  # exactly representable
    packed = W.pack_pages(kq, torch.from_numpy(scale)).numpy()
    qb = torch.from_numpy(q).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    bt = np.array([[0]], dtype=np.int32)
    sl = np.array([L], dtype=np.int32)
    exp = np.array([scale[t] * np.sum(np.maximum(k[t, :64], 0) * w[0]) for t in range(L)])
    return qb, packed, w, sl, bt, exp


@pytest.mark.parametrize("sign", [1.0, -1.0])
def test_known_answer_one_hot(oracle_mod, sign):
    q, kc, w, sl, bt, exp = _one_hot_case(sign)
    lg = oracle_mod.logits(q, kc, w, sl, bt)
    assert np.allclose(lg[0, :40], exp, rtol=1e-6, atol=0)
    assert np.all(np.isneginf(lg[0, 40:]))
    ln = oracle_mod.logits_numpy(q, kc, w, sl, bt)
    assert np.allclose(ln[0, :40], exp, rtol=1e-6, atol=0)


def test_relu_weight_order_hand_computed(oracle_mod):
    """One token, two non-zero heads: logit = scale*(ReLU(S0)*w0 + ReLU(S1)*w1)."""
    q = np.zeros((1, 64, 128), dtype=np.float32)
    q[0, 0, :4] = [1.0, 2.0, -1.0, 0.5]
    q[0, 1, :4] = [-1.0, -1.0, 1.0, 0.0]
    k = np.zeros((64, 128), dtype=np.float32)
    k[0, :4] = [2.0, 1.0, 1.0, 4.0]  # S0 = 2+2-1+2 = 5, S1 = -2-1+1 = -2 -> ReLU 0
    w = np.zeros((1, 64), dtype=np.float32)
    w[0, 0], w[0, 1] = 0.75, 10.0
    scale = np.full(64, 0.5, dtype=np.float32)
    kc = W.pack_pages(torch.from_numpy(k).to(torch.float8_e4m3fn), torch.from_numpy(scale)).numpy()
    qb = torch.from_numpy(q).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    lg = oracle_mod.logits(qb, kc, w, np.array([1], np.int32), np.array([[0]], np.int32))
    assert lg[0, 0] == np.float32(0.5 * 5 * 0.75)


def test_c_and_numpy_restatements_agree(oracle_mod):
    inp = W.make_inputs([1500, 4096, 130, 2049], seed=5)
    args = _inputs_np(inp)
    a, mag = oracle_mod.logits(*args, nthreads=4, with_mag=True)
    b = oracle_mod.logits_numpy(*args)
    fin = np.isfinite(a)
    assert np.array_equal(fin, np.isfinite(b))
    assert np.allclose(a[fin], b[fin], rtol=1e-6, atol=1e-6 * mag[fin].max())


def test_threads_do_not_change_result(oracle_mod):
    inp = W.make_inputs([3000, 777], seed=6)
    args = _inputs_np(inp)
    assert np.array_equal(oracle_mod.logits(*args, nthreads=1), oracle_mod.logits(*args, nthreads=7))


@pytest.mark.parametrize("L", [0, 1, 63, 64, 65, 2047, 2048])
def test_short_rows_token_order(oracle_mod, L):
    inp = W.make_inputs([max(L, 1)], max_pages=40, seed=L)
    d = inp.numpy()
    sl = np.array([L], np.int32)
    ids, _ = oracle_mod.run(d["q"], d["k_cache"], d["weights"], sl, d["block_table"])
    exp = np.full(TOPK, -1, np.int64)
    t = np.arange(L)
    exp[:L] = d["block_table"][0, t // 64].astype(np.int64) * 64 + t % 64
    assert np.array_equal(ids[0], exp)


def test_long_row_is_exact_topk(oracle_mod):
    inp = W.make_inputs([2049, 5000], seed=8)
    d = inp.numpy()
    ids, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    for b, L in enumerate(d["seq_lens"]):
        phys = oracle_mod.physical_ids(d["block_table"][b], L)
        order = np.argsort(-lg[b, :L], kind="stable")
        assert np.array_equal(ids[b], phys[order[:TOPK]])
    # 2049 tokens: exactly one is left out, the smallest
    left = set(oracle_mod.physical_ids(d["block_table"][0], 2049).tolist()) - set(ids[0].tolist())
    assert len(left) == 1


def test_ties_break_by_token_index(oracle_mod):
    lg = np.zeros((1, 64 * 64), dtype=np.float32)
    bt = np.arange(64, dtype=np.int32)[None, ::-1].copy()
    sl = np.array([4000], np.int32)
    ids = oracle_mod.topk(lg, sl, bt)
    assert np.array_equal(ids[0], oracle_mod.physical_ids(bt[0], 4000)[:TOPK])


def test_malformed_inputs_conventions(oracle_mod):
    inp = W.make_inputs([3000, 3000], seed=9)
    d = inp.numpy()
    bt = d["block_table"].copy()
    bt[1, 3] = 10_000_000  # out of range page -> zero page
    sl = np.array([10_000_000, 3000], np.int32)  # clamped to max_pages*64
    lg = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], sl, bt)
    assert np.isfinite(lg[0]).all()  # row 0 scored up to max_pages*64
    assert np.all(lg[1, 3 * 64:4 * 64] == 0.0)
    lg2 = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], np.array([-5, 0], np.int32), bt)
    assert np.all(np.isneginf(lg2))


def test_pairs_and_merge_equal_direct(oracle_mod):
    """A long row split into page ranges, local top-K pairs, merged: equals
    the direct top-K (random logits have no ties)."""
    inp = W.make_inputs([20000], seed=10)
    d = inp.numpy()
    ids, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    L = int(d["seq_lens"][0])
    bt = d["block_table"][0]
    for g in (2, 3, 4, 8):
        npg = (L + 63) // 64
        cuts = [npg * i // g for i in range(g + 1)]
        sc_all, tk_all = [], []
        for i in range(g):
            p0, p1 = cuts[i], cuts[i + 1]
            Li = max(0, min(L, p1 * 64) - p0 * 64)
            sub = np.full((1, (p1 - p0) * 64), -np.inf, np.float32)
            sub[0, :Li] = lg[0, p0 * 64:p0 * 64 + Li]
            sc, tk = oracle_mod.pairs(sub, np.array([Li], np.int32), token_offset=p0 * 64)
            sc_all.append(sc[0]); tk_all.append(tk[0])
        merged = oracle_mod.merge(np.concatenate(sc_all), np.concatenate(tk_all), bt, L)
        assert set(merged.tolist()) == set(ids[0].tolist())


def test_planted_tokens_rank_first(oracle_mod):
    inp = W.make_inputs([9000], seed=12)
    W.plant_tokens(inp, 0, [5, 4100, 8999])
    d = inp.numpy()
    ids, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    top3 = set(oracle_mod.physical_ids(d["block_table"][0], 9000)[[5, 4100, 8999]].tolist())
    assert top3 == set(ids[0, :3].tolist())


def test_parity_checker_catches_planted_mistakes(oracle_mod):
    inp = W.make_inputs([6000, 1000], seed=13)
    d = inp.numpy()
    ids, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    for b in range(2):
        oracle_mod.check_row(ids[b], lg[b], d["block_table"][b], int(d["seq_lens"][b]))
    # a far-from-boundary token swapped in -> rejected
    bad = ids[0].copy()
    phys = oracle_mod.physical_ids(d["block_table"][0], 6000)
    worst = phys[int(np.argmin(lg[0, :6000]))]
    bad[0] = worst
    with pytest.raises(AssertionError):
        oracle_mod.check_row(bad, lg[0], d["block_table"][0], 6000)
    # a duplicate -> rejected
    dup = ids[0].copy()
    dup[1] = dup[0]
    with pytest.raises(AssertionError):
        oracle_mod.check_row(dup, lg[0], d["block_table"][0], 6000)
    # short row off by one slot -> rejected
    short = ids[1].copy()
    short[999], short[1000] = -1, short[999]
    with pytest.raises(AssertionError):
        oracle_mod.check_row(short, lg[1], d["block_table"][1], 1000)
    # logits tolerance check rejects a 2% error
    mag = np.abs(lg[:, :]).copy()
    mag[~np.isfinite(mag)] = 0
    g = lg.copy()
    g[0, 10] *= 1.02
    with pytest.raises(AssertionError):
        oracle_mod.check_logits(g, lg, np.zeros_like(mag), d["seq_lens"])


def test_config_generators_shapes():
    inp = W.config_inputs(0)
    assert inp.rows == 2 and inp.max_pages == 64 and inp.num_pages == 88
    assert inp.seq_lens.tolist() == [1500, 4096]
    used = inp.block_table[0, :24].tolist() + inp.block_table[1, :64].tolist()
    assert sorted(used) == list(range(88))  # a permutation of the pool
    inp4 = W.make_inputs([100, 101, 102, 103, 200, 201, 202, 203], share_rows=4, seed=1)
    assert torch.equal(inp4.block_table[0], inp4.block_table[3])
    assert not torch.equal(inp4.block_table[0], inp4.block_table[4])
