import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden_paged():
    import torch
    return torch.load(GOLDEN / "paged_attention_golden.pt", weights_only=False)


@pytest.fixture(scope="session")
def golden_engine():
    import torch
    return torch.load(GOLDEN / "engine_golden.pt", weights_only=False)
