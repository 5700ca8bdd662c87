"""The int8 product's other kernels against the oracle: the int8-path product
tests and the FlowLM frame tests of test_gpu_flowlm.py rerun in a fresh
process with a switch set at initialisation — GRX_Q8_TC=1 (the tensor-core
tcgen05 kernel for every product of more than 8 rows) and GRX_Q8_G4=0 (the
mma.sync kernel with per-thread async copies for the products of 9 to 256
rows that the TMA-fed one takes by default). The fixed-scratch entry point's
tests (test_zz_no_alloc.py) rerun with them, so its 256-row product also
runs on those kernels over the library's fixed array."""

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


@pytest.mark.parametrize("switch", [("GRX_Q8_TC", "1"), ("GRX_Q8_G4", "0")])
def test_switched_int8_product_bit_exact(have_gpu, switch):
    env = dict(os.environ, **{switch[0]: switch[1]})
    r = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-x", "-p", "no:cacheprovider", "tests/test_gpu_flowlm.py",
         "tests/test_zz_no_alloc.py", "-k", "int8_path or small_frames or parts or static_scratch"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-2000:]
    assert " passed" in r.stdout and " failed" not in r.stdout
