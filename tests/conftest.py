import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG_DIR = ROOT / "deepseek-v4-a100-sglang_b200"
for p in (str(ROOT), str(PKG_DIR), str(Path(__file__).resolve().parent)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture
def golden():
    import numpy as np

    def load(name):
        return np.load(GOLDEN / f"{name}.npz")

    return load
