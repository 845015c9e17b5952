"""GPU parity of the sparse MLA attention (the consumer of the indexer's
topk_indices) against the golden vectors of the operator's published
reference definition and against the CPU oracle.

Tolerances: output (bf16) within 1e-2 + 2e-2 * |reference| (the kernel rounds
the softmax weights to bf16 for the tensor cores, the reference keeps them in
fp32); lse (base 2) within 2e-3; tokens without a valid entry exactly 0 and
-inf.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import _lib, kernel, read_attn_status, sparse_attention
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
GOLDEN = Path(__file__).resolve().parent / "golden" / "sparse_attn_golden.npz"
SCALE = 1.0 / np.sqrt(192.0)


def bf16(u16):
    return torch.from_numpy(np.asarray(u16, np.uint16).view(np.int16)).view(torch.bfloat16)


def run_gpu(qn, qp, ckv, kpe, idx, scale):
    T = qn.shape[0]
    out = torch.full((T, 16, 512), float("nan"), dtype=torch.bfloat16, device=DEV)
    lse = torch.full((T, 16), float("nan"), dtype=torch.float32, device=DEV)
    sparse_attention(qn, qp, ckv, kpe, idx, scale, out, lse)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


def check(out, lse, out_ref, lse_ref):
    assert np.all(np.isfinite(out))
    np.testing.assert_allclose(out, out_ref, rtol=2e-2, atol=1e-2)
    fin = np.isfinite(lse_ref)
    assert np.array_equal(np.isfinite(lse), fin)
    np.testing.assert_allclose(lse[fin], lse_ref[fin], rtol=0, atol=2e-3)
    assert np.all(np.isneginf(lse[~fin]))


def random_case(T, pages, seed, pattern):
    g = torch.Generator().manual_seed(seed)
    qn = torch.randn((T, 16, 512), generator=g).to(torch.bfloat16)
    qp = torch.randn((T, 16, 64), generator=g).to(torch.bfloat16)
    ckv = torch.randn((pages, 64, 512), generator=g).to(torch.bfloat16)
    kpe = torch.randn((pages, 64, 64), generator=g).to(torch.bfloat16)
    slots = pages * 64
    idx = torch.full((T, 2048), -1, dtype=torch.int32)
    for t in range(T):
        if pattern == "full":
            idx[t] = torch.randperm(slots, generator=g)[:2048].to(torch.int32)
        elif pattern == "mixed":
            n = [0, 1, 63, 64, 65, 700, 2047, 2048][t % 8]
            idx[t, :n] = torch.randperm(slots, generator=g)[:n].to(torch.int32)
            if t % 3 == 0:  # scattered padding instead of a prefix
                idx[t] = idx[t][torch.randperm(2048, generator=g)]
    return qn, qp, ckv, kpe, idx


def oracle_case(oracle_mod, qn, qp, ckv, kpe, idx, scale):
    return oracle_mod.sparse_attention(qn.float().numpy(), qp.float().numpy(), ckv.float().numpy(),
                                       kpe.float().numpy(), idx.numpy(), scale)


def test_golden_vectors():
    z = np.load(GOLDEN)
    ins = [bf16(z[k]).to(DEV) for k in ("q_nope", "q_pe", "ckv", "kpe")]
    idx = torch.from_numpy(z["sparse_indices"]).to(DEV)
    out, lse = run_gpu(*ins, idx, float(z["sm_scale"]))
    ref = bf16(z["output"]).float().numpy()
    check(out, lse, ref, z["lse"])
    assert np.all(out[2] == 0)
    assert read_attn_status(DEV) == 0


@pytest.mark.parametrize("T,pattern", [(1, "full"), (3, "mixed"), (64, "full"), (16, "mixed"), (160, "mixed")])
def test_against_oracle(oracle_mod, T, pattern):
    """T = 1, 3, 16, 64, 160 exercise 32, 32, 8, 2 and 1 splits per token."""
    qn, qp, ckv, kpe, idx = random_case(T, 64 if pattern == "mixed" else 80, 100 + T, pattern)
    out, lse = run_gpu(qn.to(DEV), qp.to(DEV), ckv.to(DEV), kpe.to(DEV), idx.to(DEV), SCALE)
    out_ref, lse_ref = oracle_case(oracle_mod, qn, qp, ckv, kpe, idx, SCALE)
    check(out, lse, out_ref, lse_ref)
    assert read_attn_status(DEV) == 0


def test_repeated_and_out_of_range_indices(oracle_mod):
    """Repeated slots count once per occurrence (as in the reference);
    indices outside [-1, slots) are treated as padding and flagged."""
    qn, qp, ckv, kpe, idx = random_case(4, 8, 7, "empty")
    g = torch.Generator().manual_seed(8)
    idx[0] = torch.randint(0, 512, (2048,), generator=g).to(torch.int32)
    idx[1, :300] = torch.randint(0, 512, (300,), generator=g).to(torch.int32)
    bad = idx.clone()
    bad[1, 300] = 512       # one past the last slot
    bad[1, 301] = -5
    out, lse = run_gpu(qn.to(DEV), qp.to(DEV), ckv.to(DEV), kpe.to(DEV), bad.to(DEV), SCALE)
    assert read_attn_status(DEV) & _lib.STATUS_BAD_INDEX
    out_ref, lse_ref = oracle_case(oracle_mod, qn, qp, ckv, kpe, idx, SCALE)
    check(out, lse, out_ref, lse_ref)


def test_consumes_indexer_output(oracle_mod):
    """The indexer's topk_indices (page*64 + slot, -1 padded) over the same
    pages feed the attention directly."""
    inp = W.make_inputs([1500, 4096, 3000, 64], seed=9)
    g = inp.to(DEV)
    ids = g.out()
    kernel(g.q, g.k_cache, g.weights, g.seq_lens, g.block_table, ids)
    P = inp.num_pages
    gen = torch.Generator().manual_seed(10)
    qn = torch.randn((4, 16, 512), generator=gen).to(torch.bfloat16)
    qp = torch.randn((4, 16, 64), generator=gen).to(torch.bfloat16)
    ckv = torch.randn((P, 64, 512), generator=gen).to(torch.bfloat16)
    kpe = torch.randn((P, 64, 64), generator=gen).to(torch.bfloat16)
    out, lse = run_gpu(qn.to(DEV), qp.to(DEV), ckv.to(DEV), kpe.to(DEV), ids, SCALE)
    out_ref, lse_ref = oracle_case(oracle_mod, qn, qp, ckv, kpe, ids.cpu(), SCALE)
    check(out, lse, out_ref, lse_ref)


def test_two_calls_and_argument_errors():
    qn, qp, ckv, kpe, idx = random_case(2, 40, 11, "full")
    args = [x.to(DEV) for x in (qn, qp, ckv, kpe, idx)]
    a = run_gpu(*args, SCALE)
    b = run_gpu(*args, SCALE)
    assert np.array_equal(a[0], b[0]) and np.array_equal(a[1], b[1])
    out = torch.empty((2, 16, 512), dtype=torch.bfloat16, device=DEV)
    lse = torch.empty((2, 16), dtype=torch.float32, device=DEV)
    with pytest.raises(RuntimeError):
        sparse_attention(args[0].float(), *args[1:], SCALE, out, lse)
    with pytest.raises(RuntimeError):
        sparse_attention(*args[:4], args[4][:, :100].contiguous(), SCALE, out, lse)
