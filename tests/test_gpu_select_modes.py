"""Both selection shapes stay under the parity tests.

A call selects with the split kernel (several CTAs per row, when one wave
of resident CTAs covers the batch) or with the one-CTA-per-row /
one-cluster-per-row kernels.  The library reads DSAI_SELECT once per
process, so this test re-runs the parity and page-range-split tests in a
child process with DSAI_SELECT=rows, where every call takes the second
shape; the parent's own run of those files covers the first.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parent.parent


def test_parity_with_row_kernels_only():
    env = dict(os.environ, DSAI_SELECT="rows")
    cmd = [sys.executable, "-m", "pytest", "-q", "-m", "gpu", "-p", "no:cacheprovider",
           str(REPO / "tests" / "test_gpu_parity.py"), str(REPO / "tests" / "test_gpu_split.py")]
    res = subprocess.run(cmd, cwd=REPO, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-2000:]
