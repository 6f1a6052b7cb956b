import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN / "golden.npz")


@pytest.fixture(scope="session")
def container_path():
    return GOLDEN / "container.q4nx"


def bf16_from_bits(bits):
    from ml_dtypes import bfloat16
    return np.ascontiguousarray(np.asarray(bits, np.uint16)).view(bfloat16)


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device, or a skip on machines without one."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
