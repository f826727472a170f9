import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built extension")
    config.addinivalue_line("markers", "multigpu: needs >= 2 GPUs")


@pytest.fixture(scope="session")
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if major != 10:
        pytest.skip(f"needs sm_100 (got sm_{major}{minor})")
    from inference_optimizations_b200._ext import ext
    ext()  # fail loudly if the extension is missing on a GPU box
    return torch.device("cuda:0")
