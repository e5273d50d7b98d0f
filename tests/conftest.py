import importlib
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

PKG_NAME = "vllm-omni-neuron_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_pkg():
    """The product package lives in a directory whose name is not a Python identifier;
    ``importlib`` imports it by that name."""
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def pkg():
    p = load_pkg()
    p.build()  # no-op when libvomni_b200.so is newer than its sources
    return p


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    d = ROOT / "tests" / "golden"

    def _load(name):
        return np.load(d / name, allow_pickle=False)

    return _load


def cuda_ok():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False


@pytest.fixture(scope="session")
def dev():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)
