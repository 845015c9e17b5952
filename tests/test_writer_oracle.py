"""CPU checks of the index-K cache writer's oracle (test infrastructure): its
e4m3 encoder against torch's float8_e4m3fn conversion, and its output
against the page format the synthetic workloads are packed in
(workloads.quantize_tokens + pack_pages), which is the format the indexer
and the reference read."""
import numpy as np
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

PAGE_BYTES = 8448


def test_e4m3_encoder_matches_torch(oracle_mod):
    rng = np.random.default_rng(5)
    edge = np.array([0.0, -0.0, 448.0, -448.0, 447.9, 416.0, 432.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10,
                     1.5 * 2.0 ** -9, 2.0 ** -6, 2.0 ** -6 * (1 - 2 ** -5), 1.0625, 1.1875, 0.001953125],
                    np.float32)
    vals = np.concatenate([rng.normal(size=4000).astype(np.float32) * np.float32(60),
                           rng.uniform(-0.02, 0.02, 2000).astype(np.float32), edge, -edge])
    ours = np.array([oracle_mod.e4m3_encode(v) for v in vals], np.uint8)
    ref = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    assert np.array_equal(ours, ref)
    # values beyond the finite range saturate to +-448
    assert oracle_mod.e4m3_encode(1000.0) == 0x7E and oracle_mod.e4m3_encode(-1e9) == 0xFE


def test_oracle_writer_reproduces_the_packed_format(oracle_mod):
    n_pages = 5
    g = torch.Generator().manual_seed(6)
    k = torch.randn((n_pages * 64, 128), generator=g) * 3
    k[7] = 0.0  # an all-zero token: scale from the 1e-12 floor
    kq, sc = W.quantize_tokens(k)
    want = W.pack_pages(kq, sc).reshape(-1).numpy()
    got = np.zeros(n_pages * PAGE_BYTES, np.uint8)
    oracle_mod.write_k(k.numpy(), np.arange(n_pages * 64, dtype=np.int32), got, n_pages)
    assert np.array_equal(got, want)


def test_oracle_writer_skips_padding_and_out_of_range_ids(oracle_mod):
    n_pages = 2
    k = np.random.default_rng(7).normal(size=(4, 128)).astype(np.float32)
    cache = np.full(n_pages * PAGE_BYTES, 0xAB, np.uint8)
    oracle_mod.write_k(k, np.array([-1, 5, 128, 1 << 20], np.int32), cache, n_pages)
    touched = np.zeros_like(cache, dtype=bool)
    touched[5 * 128:6 * 128] = True
    touched[8192 + 20:8192 + 24] = True
    assert np.all(cache[~touched] == 0xAB)
    assert not np.all(cache[touched] == 0xAB)
