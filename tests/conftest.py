import sys
from pathlib import Path

import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
sys.path.insert(0, str(Path(__file__).resolve().parent))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")
    config.addinivalue_line("markers", "multi_gpu: needs at least two GPUs")


@pytest.fixture(autouse=True)
def small_threads():
    torch.set_num_threads(1)
    torch.manual_seed(123)
