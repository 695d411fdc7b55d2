import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_ROOT = ROOT / "custom-ml-library_b200"
for path in (str(ROOT), str(PKG_ROOT)):
    if path not in sys.path:
        sys.path.insert(0, path)

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture
def golden():
    import numpy as np

    def load(name):
        with np.load(GOLDEN / f"{name}.npz") as data:
            return {k: data[k] for k in data.files}

    return load
