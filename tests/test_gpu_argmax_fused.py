"""GPU parity of the persistent fused-resolution f32 argmax kernel against
the CPU oracle, bit-exact: forced on at oracle-sized cases in a child
process, and at a size where the engine selects it by itself."""
import os
import subprocess
import sys

import numpy as np
import pytest

from helpers import engine, oracle, same_bits

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def test_fused_kernel_forced_cases():
    env = dict(os.environ, TROPICAL_GEMM_ARGMAX_FUSED="1")
    r = subprocess.run([sys.executable, os.path.join(HERE, "_fused_cases.py")], env=env, capture_output=True,
                       text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "MISMATCH" not in r.stdout and r.stdout.count(" ok") >= 20, r.stdout


def test_fused_kernel_default_selection_sampled_rows():
    """8192^3 (K >= 8192, 27.7 tiles per SM): the default dispatch takes the
    fused kernel; full rows of a sample against the oracle."""
    rng = np.random.default_rng(7)
    m, k, n = 8192, 8192, 8192
    a = rng.standard_normal((m, k), dtype=np.float32)
    b = rng.standard_normal((k, n), dtype=np.float32)
    c, am = engine("maxplus", a, b)
    rows = rng.choice(m, 24, replace=False)
    c0, am0 = oracle("maxplus", np.ascontiguousarray(a[rows]), b)
    assert same_bits(c[rows], c0) and np.array_equal(am[rows], am0)
