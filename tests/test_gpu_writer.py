"""GPU checks of the index-K cache writer (dsai_write_k / write_index_k):
bytes identical to the CPU oracle for fp32 and bf16 keys (e4m3 conversion
is round-to-nearest-even on both sides, the scale division is IEEE), ids of
-1 and out-of-range ids skipped with the rest of the cache untouched, and the
indexer run on pages the writer produced gives the same ids as on the same
pages packed on the host."""
import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import kernel, write_index_k
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
PAGE_BYTES = 8448


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_writer_matches_oracle(oracle_mod, dtype):
    n_pages, n = 40, 1500
    rng = np.random.default_rng(11)
    k = torch.from_numpy(rng.normal(size=(n, 128)).astype(np.float32) * 5).to(dtype)
    k[3] = 0
    k[4, :64] = -0.0                    # signed zeros keep their sign
    ids = rng.permutation(n_pages * 64)[:n].astype(np.int32)
    ids[::37] = -1                      # padding
    ids[5] = n_pages * 64 + 3           # out of range
    init = rng.integers(0, 256, n_pages * PAGE_BYTES, dtype=np.uint8)
    cache = torch.from_numpy(init.copy()).to(DEV).view(n_pages, 64, 1, 132)
    write_index_k(k.to(DEV), torch.from_numpy(ids).to(DEV), cache)
    torch.cuda.synchronize()
    want = init.copy()
    oracle_mod.write_k(k.float().numpy(), ids, want, n_pages)
    assert np.array_equal(cache.reshape(-1).cpu().numpy(), want)


def test_writer_empty_and_argument_errors():
    cache = torch.zeros((2, 64, 1, 132), dtype=torch.uint8, device=DEV)
    write_index_k(torch.empty((0, 128), device=DEV), torch.empty(0, dtype=torch.int32, device=DEV), cache)
    assert int(cache.sum()) == 0
    with pytest.raises(RuntimeError):
        write_index_k(torch.zeros((4, 128), dtype=torch.float16, device=DEV),
                      torch.zeros(4, dtype=torch.int32, device=DEV), cache)
    with pytest.raises(RuntimeError):
        write_index_k(torch.zeros((4, 64), device=DEV), torch.zeros(4, dtype=torch.int32, device=DEV), cache)


def test_indexer_reads_what_the_writer_wrote(oracle_mod):
    """A batch's keys written in shuffled order by the GPU writer give the
    bytes of the CPU writer, and the indexer's ids on those pages agree with
    the oracle's."""
    lens = [9000, 3000, 1200]
    inp = W.make_inputs(lens, seed=12)
    kq, sc = W.unpack_pages(inp.k_cache)
    k_deq = (kq.float() * sc.unsqueeze(-1)).reshape(-1, 128)  # the batch's keys, dequantised
    pool = torch.zeros_like(inp.k_cache).to(DEV)
    ids = torch.arange(k_deq.shape[0], dtype=torch.int32)
    perm = torch.randperm(k_deq.shape[0], generator=torch.Generator().manual_seed(3))
    write_index_k(k_deq[perm].to(DEV), ids[perm].to(DEV), pool)
    want = inp.k_cache.clone().reshape(-1).numpy()
    oracle_mod.write_k(k_deq.numpy(), ids.numpy(), want, inp.num_pages)
    got = pool.reshape(-1).cpu().numpy()
    assert np.array_equal(got, want)
    g = inp.to(DEV)
    out = g.out()
    kernel(g.q, pool, g.weights, g.seq_lens, g.block_table, out)
    torch.cuda.synchronize()
    d = inp.numpy()
    d["k_cache"] = got.reshape(d["k_cache"].shape)
    exp, lg = oracle_mod.run(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"])
    res = out.cpu().numpy()
    for b, L in enumerate(lens):
        oracle_mod.check_row(res[b], lg[b], d["block_table"][b], L)  # raises on a mismatch
