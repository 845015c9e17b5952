"""The CPU oracle against the output of the reference's own CUDA kernel.

tests/golden/reference_kernel_golden.npz holds the top-2048 ids that the
reference's kernel (solution/cuda/kernel.cu, built unmodified by
baseline/Makefile, run on a B200 by tests/golden/make_reference_kernel_
golden.py) wrote for seeded inputs.  The inputs are regenerated here (their
SHA-256 must match) and the oracle's exact top-2048 must agree with the
reference's ids: rows with seq_len <= 2048 and the -1 padding bit for bit,
longer rows as sets except among tokens that tie the 2048th logit after the
reference's fp16 rounding (oracle.REFERENCE_FP16_RTOL); those differences
are counted.  This pins the oracle, and through it every GPU parity test,
to the reference itself.
"""
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
NPZ = GOLDEN / "reference_kernel_golden.npz"
# The same cases through the reference's active path (solution/python/kernel.cu,
# baseline/build_active_variant.py), when its outputs have been generated.
NPZ_ACTIVE = GOLDEN / "reference_kernel_active_golden.npz"


def _cases():
    sys.path.insert(0, str(GOLDEN))
    import make_reference_kernel_golden as G
    return G


@pytest.mark.parametrize("npz", [NPZ, NPZ_ACTIVE], ids=["tvm_ffi_variant", "active_variant"])
def test_oracle_matches_reference_kernel_outputs(oracle_mod, npz):
    if not npz.exists():
        pytest.skip(f"{npz.name} not generated")
    G = _cases()
    z = np.load(npz)
    total_diff = 0
    rows_checked = 0
    for name, inp in G.cases().items():
        assert G.digest(inp) == str(z[f"{name}_sha256"]), f"{name}: input generator drifted"
        ref_ids = z[f"{name}_ids"]
        d = inp.numpy()
        lg = oracle_mod.logits(d["q"], d["k_cache"], d["weights"], d["seq_lens"], d["block_table"],
                               num_pages=d["num_pages"], nthreads=8)
        exact = oracle_mod.topk(lg, d["seq_lens"], d["block_table"])
        for b in range(inp.rows):
            L = int(d["seq_lens"][b])
            # the reference's row is a valid top-K in the fp16 band of the exact one
            oracle_mod.check_row(ref_ids[b], lg[b], d["block_table"][b], L, rtol=oracle_mod.REFERENCE_FP16_RTOL)
            total_diff += oracle_mod.set_diff_in_band(exact[b], ref_ids[b], lg[b], d["block_table"][b], L)
            rows_checked += 1
        if name != "ties":
            # planted / ordinary rows: the sets agree except for a few fp16 ties
            for b in range(inp.rows):
                if int(d["seq_lens"][b]) > 2048:
                    assert len(set(ref_ids[b].tolist()) & set(exact[b].tolist())) >= 2048 - 64, f"{name} row {b}"
    print(f"{npz.name} vs oracle: {rows_checked} rows, {total_diff} ids differ inside the fp16 tie band")
