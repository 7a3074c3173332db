"""pytest setup: the `gpu` marker and import paths.

`-m "not gpu"` runs on a CPU-only machine (oracle vs golden vectors, host logic, C-ABI
loading and validation). `-m gpu` needs a B200 and runs the kernel parity tests.
"""

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "flash-attention-from-scratch_b200"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a B200)")


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return REPO / "tests" / "golden"
