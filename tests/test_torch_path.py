"""The torch CPU formulation of the indexer (oracle/torch_path.py, the CPU
baseline of bench.py) against the exact C oracle: logits within 1e-5
relative (plus 1e-6 of the head-sum magnitude), ids under the north-star
parity rules."""
import numpy as np

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W
from oracle import torch_path


def test_torch_path_matches_oracle(oracle_mod):
    inp = W.make_inputs([1500, 4096, 9001, 2049, 0, 20000], seed=81)
    d = inp.numpy()
    ids, lgs = torch_path.indexer(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                                  return_logits=True)
    ora, mag = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                                 num_pages=d["num_pages"], nthreads=4, with_mag=True)
    for b in range(inp.rows):
        L = int(d["seq_lens"][b])
        if lgs[b] is not None:
            err = np.abs(lgs[b] - ora[b, :L])
            assert np.all(err <= 1e-5 * np.abs(ora[b, :L]) + 1e-6 * mag[b, :L])
        oracle_mod.check_row(ids[b], ora[b], d["block_table"][b], L)
