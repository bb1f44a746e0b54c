import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU; run with -m gpu")
    config.addinivalue_line("markers", "slow: long-running CPU oracle case")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN / "reference_vectors.npz")


@pytest.fixture(scope="session")
def golden_meta():
    return json.loads((GOLDEN / "reference_vectors.json").read_text())


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device for gpu-marked tests.  A gpu test on a host without a
    usable GPU fails instead of skipping, so a GPU run can never pass on a
    silent fallback."""
    import torch

    assert torch.cuda.is_available(), "gpu test needs a CUDA device"
    from qwen3x_b200 import capi

    capi.lib()  # raises if libq3xk.so is missing
    return torch.device("cuda:0")
