import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

from flashattentionanycard_b200.tuner.hardware import Hardware  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires an sm_100 (B200) CUDA device")


@pytest.fixture
def hardware():
    return Hardware("CPU test double; not a GPU measurement", (10, 0), 148, 180 * 1024**3, 227 * 1024)


@pytest.fixture(scope="session")
def cuda_device():
    """The sm_100 device GPU tests run on (BO_TEST_CUDA_DEVICE, default 0).

    On a machine without one this fails instead of skipping: a GPU test that
    passes by skipping would hide a missing native path."""
    import torch

    device = int(os.environ.get("BO_TEST_CUDA_DEVICE", "0"))
    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    major, _ = torch.cuda.get_device_capability(device)
    if major != 10:
        pytest.fail(f"GPU tests need an sm_100 device; device {device} is sm_{major}x")
    torch.cuda.set_device(device)
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    return torch.device(f"cuda:{device}")
