import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA path against the oracle")


@pytest.fixture(scope="session")
def have_gpu():
    import gorelaxor_b200 as g

    if g.device_count() < 1:
        pytest.skip("no CUDA device")
    return True
