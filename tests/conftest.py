from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden" / "reference_outputs.pt"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")


@pytest.fixture(scope="session")
def pkg():
    import __graft_entry__

    return __graft_entry__.load_package()


@pytest.fixture(scope="session")
def golden():
    import torch

    return torch.load(GOLDEN, weights_only=True)["cases"]


@pytest.fixture(scope="session")
def cuda_pkg(pkg):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    pkg._lib.load()
    return pkg
