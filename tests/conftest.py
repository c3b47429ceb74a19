import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

CACHE = Path(os.environ.get("MMC_TEST_CACHE", "/tmp/mmc_test_models"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) GPU")


def gpu_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def model_dir():
    """Factory: model_dir(shape, seed, eps=1e-5, theta=1e6) -> path of a seeded runtime model."""
    from minimind_orangepi_b200.synthetic import write_runtime_model

    def make(shape: str, seed: int = 1, eps=1e-5, theta=1e6):
        return write_runtime_model(CACHE / f"{shape}-s{seed}-e{eps}-t{theta}", shape, seed, eps=eps, theta=theta)

    return make
