import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")
    config.addinivalue_line("markers", "slow: long CPU case")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(ROOT / "tests" / "golden" / "reference_golden.npz"))


@pytest.fixture(scope="session")
def golden_host():
    import json
    return json.loads((ROOT / "tests" / "golden" / "reference_host.json").read_text())
