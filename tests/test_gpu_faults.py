"""Failure detection on the GPU without a fault: a kernel waits on an on-chip
barrier that nothing completes; its bounded wait gives up after a short
limit, the status word says so, and the context keeps working."""
import ctypes

import pytest
import torch

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import _lib, kernel
from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_bounded_wait_reports_timeout_and_context_survives():
    lib = _lib.load_library()
    stream = torch.cuda.current_stream(DEV).cuda_stream
    ws = _lib.Workspace(DEV)
    ptr, _ = ws.get(1, 1, stream)
    assert ws.read_status(stream) == 0
    rc = lib.dsai_selftest_wait_timeout(ptr, 2_000_000, stream)  # 2 ms
    assert rc == 0, lib.dsai_last_error()
    assert ws.read_status(stream) == _lib.STATUS_WAIT_TIMEOUT
    assert ws.read_status(stream) == 0  # reading clears
    # the context still runs the indexer
    inp = W.config_inputs(0).to(DEV)
    out = inp.out()
    kernel(inp.q, inp.k_cache, inp.weights, inp.seq_lens, inp.block_table, out)
    torch.cuda.synchronize()
    assert (out[0, 1500:] == -1).all() and (out[1] >= 0).all()


def test_selftest_rejects_unbounded_timeouts():
    lib = _lib.load_library()
    assert lib.dsai_selftest_wait_timeout(None, 1000, None) == -1
    ws = torch.empty(256, dtype=torch.uint8, device=DEV)
    assert lib.dsai_selftest_wait_timeout(ws.data_ptr(), 0, None) == -1
    assert lib.dsai_selftest_wait_timeout(ws.data_ptr(), 10 ** 12, None) == -1
