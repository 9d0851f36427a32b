"""Test configuration: import paths, the ``gpu`` marker, golden fixtures."""

import json
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "kv-block-mass_b200"))
sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) device")
    config.addinivalue_line("markers", "slow: long-running (full-size workloads)")


def load_golden(name: str):
    p = GOLDEN / f"{name}.json"
    if not p.exists():
        return None
    return json.loads(p.read_text())


@pytest.fixture(scope="session")
def small_cases():
    return load_golden("small_cases")["cases"]


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        # GPU tests run only under `-m gpu` on a B200 box; a missing device
        # there is a failure, not a skip.
        pytest.fail("gpu-marked test but torch.cuda.is_available() is False")
    return torch.device("cuda", 0)
