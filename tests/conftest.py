import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def from_bits(a: np.ndarray) -> torch.Tensor:
    """bf16 tensor from the int16 bit patterns stored in the fixtures."""
    return torch.from_numpy(a.copy()).view(torch.bfloat16)


@pytest.fixture(scope="session")
def fa_golden():
    return dict(np.load(GOLDEN / "fa_ref_cases.npz"))


@pytest.fixture(scope="session")
def smollm_golden():
    return dict(np.load(GOLDEN / "smollm_logits.npz"))


@pytest.fixture(scope="session")
def cuda_dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.skip(f"needs sm_100 (B200), found sm_{major}{minor}")
    return torch.device("cuda", 0)
