"""B200-native (sm_100a) DSA lightning indexer: FP8 scoring of a paged
index-K cache on tcgen05 tensor cores and exact top-2048 selection.

Drop-in entry point: ``kernel(q_index_fp8, k_index_cache_fp8, weights,
seq_lens, block_table, topk_indices)`` — the signature of the reference's
``solution.py::kernel``.  ``write_index_k`` fills the index-K cache it reads.
"""
from .solution import (IndexerGraph, kernel, merge_pairs, read_attn_status, read_status, run, run_pairs,  # noqa: F401
                       sparse_attention, write_index_k)

__version__ = "0.1.0"
