"""The tensor-core (tcgen05) int8 product, switched on with GRX_Q8_TC=1 at
initialisation, against the oracle: the int8-path product tests and the
FlowLM frame tests of test_gpu_flowlm.py rerun in a fresh process with the
switch set, so every int8 product of more than 8 rows goes through it."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_tensor_core_int8_product_bit_exact(have_gpu):
    env = dict(os.environ, GRX_Q8_TC="1")
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "tests/test_gpu_flowlm.py", "-k",
         "int8_path or small_frames or parts"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and " failed" not in r.stdout
