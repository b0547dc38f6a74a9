import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) CUDA device")


@pytest.fixture(scope="session")
def golden_hashes():
    return json.loads((GOLDEN / "golden_hashes.json").read_text())


@pytest.fixture(scope="session")
def golden_small():
    with np.load(GOLDEN / "golden_small.npz") as z:
        return {k: z[k] for k in z.files}
