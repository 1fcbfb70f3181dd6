import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT, ROOT / "spark-h3_b200"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA GPU (run it with -m gpu on a B200)")
    major, minor = torch.cuda.get_device_capability()
    if (major, minor) != (10, 0):
        pytest.fail(f"this test needs an sm_100 GPU, found sm_{major}{minor}")
    return torch.device("cuda", 0)
