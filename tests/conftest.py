import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs at least one CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA GPUs")


def _gpu_count() -> int:
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.fixture(scope="session")
def gpu_count():
    return _gpu_count()


@pytest.fixture(scope="session")
def native():
    from pcie_pool_b200._native import native as load

    return load()


@pytest.fixture
def need_gpu(gpu_count):
    if gpu_count < 1:
        pytest.fail("GPU test selected but no CUDA device is visible")


@pytest.fixture
def need_two_gpus(gpu_count):
    if gpu_count < 2:
        pytest.skip("needs at least two GPUs")
