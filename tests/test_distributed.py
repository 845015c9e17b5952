"""CPU tests of the multi-GPU host logic: row sharding, page ranges, and the
page-range split of one long row with its all-gather merge, run on two
``gloo`` ranks with the CPU oracle as the local compute (the CUDA entry points
replace it on GPUs; their parity is covered by the GPU tests)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import distributed as D
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

TOPK = 2048


def test_shard_rows_cover_and_balance():
    sl = np.array([4000, 30000, 5000, 5000, 29000, 100, 0, 12000])
    for world in (1, 2, 3, 4, 8):
        spans = [D.shard_rows(sl, world, r) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == len(sl)
        for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
            assert a1 == b0 and a0 <= a1
    # balanced by tokens: no rank gets more than its share plus one row
    spans = [D.shard_rows(sl, 2, r) for r in range(2)]
    tok = [sl[a:b].sum() for a, b in spans]
    assert max(tok) - min(tok) <= sl.max()


def test_page_ranges_partition_the_row():
    for L in (0, 1, 64, 65, 4096, 131072, 131071):
        for world in (1, 2, 3, 8):
            pr = [D.page_range(L, world, r) for r in range(world)]
            assert pr[0][0] == 0 and pr[-1][1] == (L + 63) // 64
            assert all(a[1] == b[0] for a, b in zip(pr, pr[1:]))


def _oracle_local_pairs(oracle):
    def local_pairs(q_row, k_cache, weights_row, seq_len_local, bt_local, token_offset):
        if bt_local.shape[1] == 0:
            return torch.full((TOPK,), float("-inf")), torch.full((TOPK,), -1, dtype=torch.int32)
        q = q_row.view(torch.uint8).numpy()
        lg = oracle.logits(q, k_cache.numpy(), weights_row.numpy(), np.array([seq_len_local], np.int32),
                           bt_local.numpy())
        sc, tk = oracle.pairs(lg, np.array([seq_len_local], np.int32), token_offset)
        return torch.from_numpy(sc[0]), torch.from_numpy(tk[0])
    return local_pairs


def _oracle_merge(oracle):
    def merge(scores, tokens, bt_row_full, seq_len, out):
        out.copy_(torch.from_numpy(oracle.merge(scores.numpy(), tokens.numpy(), bt_row_full.numpy(), seq_len)))
    return merge


def _worker(rank, world, port, seq_len, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import oracle
        inp = W.make_inputs([seq_len], seed=77)
        W.plant_tokens(inp, 0, [3, seq_len // 2 - 1, seq_len // 2, seq_len - 1])
        p0, p1 = D.page_range(seq_len, world, rank)
        out = torch.full((TOPK,), -7, dtype=torch.int32)
        D.split_row_topk(inp.q, inp.k_cache, inp.weights, seq_len, inp.block_table[0, p0:p1],
                         inp.block_table[0], out, local_pairs=_oracle_local_pairs(oracle),
                         merge=_oracle_merge(oracle))
        result_q.put((rank, out.numpy().copy()))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("seq_len,world", [(9000, 2), (1500, 2), (9000, 4)])
def test_split_row_on_gloo_ranks_matches_direct(oracle_mod, seq_len, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seq_len, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    inp = W.make_inputs([seq_len], seed=77)
    W.plant_tokens(inp, 0, [3, seq_len // 2 - 1, seq_len // 2, seq_len - 1])
    d = inp.numpy()
    direct, _ = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    for r in range(world):
        assert np.array_equal(results[r], results[0])  # every rank holds the merged result
        if seq_len <= TOPK:
            assert np.array_equal(results[r], direct[0])
        else:
            assert set(results[r].tolist()) == set(direct[0].tolist())
    planted = oracle_mod.physical_ids(d["block_table"][0], seq_len)[[3, seq_len // 2 - 1, seq_len // 2, seq_len - 1]]
    assert set(planted.tolist()) <= set(results[0].tolist())


def _gather_worker(rank, world, port, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        counts = [3, 2, 0, 1][:world]
        local = torch.arange(counts[rank] * TOPK, dtype=torch.int32).view(counts[rank], TOPK) + 100000 * rank
        buf = torch.empty((world, max(counts), TOPK), dtype=torch.int32)
        got = D.gather_rows(local, counts, buf=buf)
        got2 = D.gather_rows(local, counts)  # without a caller buffer
        result_q.put((rank, got.numpy().copy(), got2.numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gather_rows_on_gloo_ranks(world):
    """Rows sharded unevenly (3, 2, 0 and 1 rows): every rank gets all rows
    in rank order."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, a, b = q.get(timeout=120)
        results[r] = (a, b)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    counts = [3, 2, 0, 1][:world]
    exp = np.concatenate([np.arange(c * TOPK, dtype=np.int32).reshape(c, TOPK) + 100000 * g
                          for g, c in enumerate(counts)])
    for r in range(world):
        assert np.array_equal(results[r][0], exp) and np.array_equal(results[r][1], exp)
