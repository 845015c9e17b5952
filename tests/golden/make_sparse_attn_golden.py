"""Generates tests/golden/sparse_attn_golden.npz: seeded inputs of the DSA
sparse MLA attention (16 heads, ckv 512, kpe 64, top-2048, page 64) and the
outputs of the operator's published reference definition in flashinfer
0.6.11.post2 (flashinfer.trace.templates.attention._dsa_paged_reference),
run on the CPU.  bf16 tensors are stored as their uint16 bit patterns.

Run once where flashinfer is importable:  python tests/golden/make_sparse_attn_golden.py
"""
import math
from pathlib import Path

import numpy as np
import torch

from flashinfer.trace.templates.attention import _dsa_paged_reference


def main():
    g = torch.Generator().manual_seed(2026)
    T, H, D, DP, PAGES, PS, TOPK = 5, 16, 512, 64, 4, 64, 2048
    slots = PAGES * PS
    q_nope = torch.randn((T, H, D), generator=g).to(torch.bfloat16)
    q_pe = torch.randn((T, H, DP), generator=g).to(torch.bfloat16)
    ckv = torch.randn((PAGES, PS, D), generator=g).to(torch.bfloat16)
    kpe = torch.randn((PAGES, PS, DP), generator=g).to(torch.bfloat16)
    idx = torch.full((T, TOPK), -1, dtype=torch.int32)
    idx[0, :slots] = torch.randperm(slots, generator=g).to(torch.int32)           # every slot once, then padding
    idx[1, :100] = torch.randperm(slots, generator=g)[:100].to(torch.int32)       # a short prefix
    # row 2: no valid entry (output 0, lse -inf)
    idx[3] = torch.randint(0, slots, (TOPK,), generator=g).to(torch.int32)        # full row, repeated slots
    sel = torch.randperm(TOPK, generator=g)[:700]                                  # valid entries scattered
    idx[4, sel] = torch.randint(0, slots, (700,), generator=g).to(torch.int32)
    sm_scale = 1.0 / math.sqrt(128 + 64)
    out, lse = _dsa_paged_reference(q_nope, q_pe, ckv, kpe, idx, sm_scale)
    u16 = lambda x: x.contiguous().view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(Path(__file__).with_name("sparse_attn_golden.npz"),
                        q_nope=u16(q_nope), q_pe=u16(q_pe), ckv=u16(ckv), kpe=u16(kpe),
                        sparse_indices=idx.numpy(), sm_scale=np.float32(sm_scale),
                        output=u16(out), lse=lse.numpy())


if __name__ == "__main__":
    main()
