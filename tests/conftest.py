import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    from oracle_lib import Oracle

    return Oracle.load()


@pytest.fixture(scope="session")
def gpu_lib():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu-marked test needs a CUDA device")
    from confkv_b200 import build
    from confkv_b200.gpu_aesgcm import GpuAesGcmLibrary

    build.build()
    return GpuAesGcmLibrary()


@pytest.fixture(scope="session")
def cpu_lib():
    """The product library loaded without touching a GPU (ABI checks only)."""
    from confkv_b200 import build
    from confkv_b200.gpu_aesgcm import GpuAesGcmLibrary

    build.build()
    return GpuAesGcmLibrary()


@pytest.fixture(autouse=True)
def _no_alloc_fault_env():
    for name in ("CONFKV_B200_FAIL_ALLOC", "CONFKV_B200_TEST_HANDOFF_STALL"):
        os.environ.pop(name, None)
    yield
    for name in ("CONFKV_B200_FAIL_ALLOC", "CONFKV_B200_TEST_HANDOFF_STALL"):
        os.environ.pop(name, None)
