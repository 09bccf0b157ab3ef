"""Shared pytest setup: the `gpu` marker, import paths, golden fixtures."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for _p in (str(ROOT / "python"), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_vectors.pt"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def golden_cases():
    import torch
    return torch.load(GOLDEN, weights_only=False)["cases"]


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    assert torch.cuda.is_available(), "GPU test run without a CUDA device"
    major, minor = torch.cuda.get_device_capability(0)
    assert (major, minor) == (10, 0), f"needs sm_100 (B200), found sm_{major}{minor}"
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def ext():
    """The package, imported (which loads the extension modules)."""
    import esimd_learning_b200
    return esimd_learning_b200
