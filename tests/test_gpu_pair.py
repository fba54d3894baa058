"""GPU: the prefill kernel on CTA pairs (cta_group::2, 256-row tiles). By default the library uses it for the
fused kernel from 1024 rows only; here the prefill GEMM and fused cases of test_gpu_kernels.py run again in a
child process with BS_FP8_PAIR_MIN_ROWS=512, so every pair tile shape there (full, last tile with 8 valid rows,
last tile whose second CTA holds no valid row, half-empty last column tile) and the plain GEMM on pairs are
checked against the oracle."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def test_pair_prefill_matches_oracle():
    env = dict(os.environ, BS_FP8_PAIR_MIN_ROWS="512")
    cmd = [sys.executable, "-m", "pytest", str(ROOT / "tests" / "test_gpu_kernels.py"), "-q", "-x", "-m", "gpu",
           "-k", "1024 or 600 or 520 or 1000", "-p", "no:cacheprovider"]
    proc = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-2000:]
    assert " passed" in proc.stdout and "deselected" in proc.stdout
