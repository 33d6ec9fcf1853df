import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def orc():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("models"))


@pytest.fixture(scope="session")
def cuda():
    """torch on cuda:0 plus an initialised liblmc_b200 (GPU tests only)."""
    import torch
    from lmc_b200 import runtime
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    torch.cuda.set_device(0)
    runtime.init(0)
    return torch


def rel_err(a, b):
    """Norm-wise relative error ||a - b|| / ||b|| (the rel-err 1e-3 bar)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
