"""CPU test of the launch recorder behind the graph cache (csrc/graph.h):
a small host program (tests/native/graph_record_test.cu) records launches
through launch_kernel() and checks the recorded kernels, launch
configurations, attributes and argument bytes.  Built with nvcc, run on the
host (it makes no CUDA call, so it needs no GPU)."""
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
CSRC = REPO / "dsa_topk_indexer_fp8_h64_d128_topk2048_ps64_b200" / "csrc"


def test_launch_recorder(tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(nvcc).exists():
        pytest.skip("nvcc unavailable")
    exe = tmp_path / "graph_record_test"
    build = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-std=c++17", "-O1",
                            "-I", str(CSRC), "-o", str(exe), str(REPO / "tests" / "native" / "graph_record_test.cu"),
                            str(CSRC / "graph.cu")], capture_output=True, text=True, timeout=300)
    assert build.returncode == 0, build.stderr[-2000:]
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0 and run.stdout.strip() == "ok", run.stdout + run.stderr
