"""CPU tests of the C ABI: the library loads without a GPU, exports every
function include/dsai.h declares, sizes its workspace, and rejects bad
arguments before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import _lib

HEADER = Path(__file__).resolve().parent.parent / "include" / "dsai.h"


def declared_functions():
    text = HEADER.read_text()
    return re.findall(r"DSAI_API\s+[\w\s\*]+?\b(dsai_\w+)\s*\(", text)


def test_header_declares_the_api():
    names = declared_functions()
    assert set(names) == set(_lib.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol(dsai_lib):
    for name in declared_functions():
        assert hasattr(dsai_lib, name), name
    assert dsai_lib.dsai_version().decode().startswith("dsai")


def test_only_the_api_is_exported(dsai_lib):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True)
    if out.returncode != 0:
        pytest.skip("nm unavailable")
    exported = {l.split()[-1] for l in out.stdout.splitlines() if " T " in l}
    dsai = {s for s in exported if s.startswith("dsai_")}
    assert dsai == set(_lib.EXPORTED_SYMBOLS)


def test_workspace_size(dsai_lib):
    # header + per row a 4096-bin u32 histogram with 4 u32 counters (256-B
    # rounded) + per row a 4096-entry (key, value) list + fp32 logits (256-B rounded)
    def r256(n):
        return (n + 255) // 256 * 256
    assert dsai_lib.dsai_workspace_size(0, 0) == 256
    assert dsai_lib.dsai_workspace_size(64, 512) == 256 + r256(64 * 16400) + 64 * 32768 + 64 * 512 * 64 * 4
    assert dsai_lib.dsai_workspace_size(3, 5) == 256 + r256(3 * 16400) + 3 * 32768 + r256(3 * 5 * 64 * 4)
    assert dsai_lib.dsai_workspace_size(-1, 4) == 0


def _args(**kw):
    a = _lib.DsaiArgs()
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_run_rejects_bad_arguments_without_device(dsai_lib):
    assert dsai_lib.dsai_run(None, None, 0, None) == -1
    assert b"NULL" in dsai_lib.dsai_last_error()
    a = _args(rows=-2, max_pages=4, num_pages=4)
    assert dsai_lib.dsai_run(ctypes.byref(a), None, 0, None) == -1
    assert b"negative" in dsai_lib.dsai_last_error()
    # zero rows is a no-op success
    a = _args(rows=0, max_pages=4, num_pages=4)
    assert dsai_lib.dsai_run(ctypes.byref(a), None, 0, None) == 0
    # missing workspace / too small / misaligned
    a = _args(rows=2, max_pages=4, num_pages=4, seq_lens=16, block_table=32, topk_indices=64)
    assert dsai_lib.dsai_run(ctypes.byref(a), None, 0, None) == -2
    assert dsai_lib.dsai_run(ctypes.byref(a), 256, 16, None) == -2
    assert b"too small" in dsai_lib.dsai_last_error()
    assert dsai_lib.dsai_run(ctypes.byref(a), 300, 1 << 20, None) == -2
    assert b"aligned" in dsai_lib.dsai_last_error()
    a = _args(rows=2, max_pages=4, num_pages=4, seq_lens=16, block_table=32, topk_indices=68)
    assert dsai_lib.dsai_run(ctypes.byref(a), 256, 1 << 20, None) == -1
    a = _args(rows=2, max_pages=4, num_pages=4, seq_lens=None, block_table=32, topk_indices=64)
    assert dsai_lib.dsai_run(ctypes.byref(a), 256, 1 << 20, None) == -1


def test_rows_per_seq_checked_without_device(dsai_lib):
    for rows, rps in ((3, 2), (8, 5), (8, -1)):
        a = _args(rows=rows, max_pages=4, num_pages=4, seq_lens=16, block_table=32, topk_indices=64,
                  rows_per_seq=rps)
        assert dsai_lib.dsai_run(ctypes.byref(a), 256, 1 << 20, None) == _lib.E_INVALID
        assert b"rows_per_seq" in dsai_lib.dsai_last_error()


def test_args_struct_layout_matches_header(tmp_path):
    """The ctypes mirror of dsai_args has the C struct's size and offsets."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f[0] for f in _lib.DsaiArgs._fields_]
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "dsai.h"', "int main(void) {"]
    lines += [f'  printf("%zu\\n", offsetof(dsai_args, {f}));' for f in fields]
    lines += ['  printf("%zu\\n", sizeof(dsai_args));', "  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [getattr(_lib.DsaiArgs, f).offset for f in fields] + [ctypes.sizeof(_lib.DsaiArgs)]
    assert got == want


def test_sparse_attn_checked_without_device(dsai_lib):
    """The sparse attention validates its arguments before it touches the
    device; its workspace is a 256-B header at least."""
    assert dsai_lib.dsai_sparse_attn(None, None, 0, None) == _lib.E_INVALID
    a = _lib.DsaiAttnArgs(num_tokens=0, num_pages=4)
    assert dsai_lib.dsai_sparse_attn(ctypes.byref(a), None, 0, None) == 0  # nothing to do
    a = _lib.DsaiAttnArgs(num_tokens=-1, num_pages=4)
    assert dsai_lib.dsai_sparse_attn(ctypes.byref(a), None, 0, None) == _lib.E_INVALID
    a = _lib.DsaiAttnArgs(num_tokens=70000, num_pages=4)
    assert dsai_lib.dsai_sparse_attn(ctypes.byref(a), None, 0, None) == _lib.E_INVALID
    assert b"65535" in dsai_lib.dsai_last_error()
    a = _lib.DsaiAttnArgs(q_nope=16, q_pe=32, ckv_cache=48, kpe_cache=None, sparse_indices=64, output=80, lse=96,
                          sm_scale=0.1, num_tokens=2, num_pages=4)
    assert dsai_lib.dsai_sparse_attn(ctypes.byref(a), 256, 1 << 20, None) == _lib.E_INVALID
    assert b"NULL" in dsai_lib.dsai_last_error()
    a.kpe_cache, a.q_pe = 64, 40  # q_pe not 16-B aligned
    assert dsai_lib.dsai_sparse_attn(ctypes.byref(a), 256, 1 << 20, None) == _lib.E_INVALID
    a.q_pe, a.sm_scale = 32, float("inf")
    assert dsai_lib.dsai_sparse_attn(ctypes.byref(a), 256, 1 << 20, None) == _lib.E_INVALID
    a.sm_scale = 0.1
    assert dsai_lib.dsai_sparse_attn(ctypes.byref(a), 300, 1 << 20, None) == _lib.E_WORKSPACE
    assert dsai_lib.dsai_sparse_attn_workspace_size(-1) == 0
    assert dsai_lib.dsai_sparse_attn_workspace_size(0) >= 256


def test_attn_args_struct_layout_matches_header(tmp_path):
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f[0] for f in _lib.DsaiAttnArgs._fields_]
    lines = ["#include <stdio.h>", "#include <stddef.h>", '#include "dsai.h"', "int main(void) {"]
    lines += [f'  printf("%zu\\n", offsetof(dsai_attn_args, {f}));' for f in fields]
    lines += ['  printf("%zu\\n", sizeof(dsai_attn_args));', "  return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert got == [getattr(_lib.DsaiAttnArgs, f).offset for f in fields] + [ctypes.sizeof(_lib.DsaiAttnArgs)]


def test_merge_and_status_reject_null(dsai_lib):
    assert dsai_lib.dsai_merge_pairs(None, None, -1, None, 4, None, None, None) == -1
    assert dsai_lib.dsai_merge_pairs(None, None, 4, 16, 4, 16, 16, None) == -1
    assert dsai_lib.dsai_read_status(None, None, None) == -1


def test_python_entry_validates_like_the_reference():
    """The drop-in raises RuntimeError for non-CUDA / wrong-dtype tensors, as
    the reference's TORCH_CHECKs do."""
    import torch
    from dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200 import kernel
    bt = torch.zeros((2, 4), dtype=torch.int32)
    sl = torch.zeros(2, dtype=torch.int32)
    out = torch.zeros((2, 2048), dtype=torch.int32)
    with pytest.raises(RuntimeError, match="block_table must be int32 contiguous CUDA"):
        kernel(None, None, None, sl, bt, out)


def test_noalloc_rejects_without_device(dsai_lib):
    """The allocation-free entry point checks its arguments and its size
    limit before it touches the device."""
    assert dsai_lib.dsai_run_noalloc(None, None) == -1
    a = _args(rows=256, max_pages=2048, num_pages=1)  # far more than its 16 MiB array
    assert dsai_lib.dsai_run_noalloc(ctypes.byref(a), None) == -2
    assert b"static scratch" in dsai_lib.dsai_last_error()
    for bad in (dict(rows=-1, max_pages=4, num_pages=1), dict(rows=2, max_pages=-4, num_pages=1),
                dict(rows=2, max_pages=4, num_pages=-1)):
        assert dsai_lib.dsai_run_noalloc(ctypes.byref(_args(**bad)), None) == -1
        assert b"negative size" in dsai_lib.dsai_last_error()
    assert dsai_lib.dsai_noalloc_read_status(None, None) == -1
