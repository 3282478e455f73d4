import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "lemon-mlx-engine_b200")
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA path)")


def load_lmx():
    """Import the package's ctypes binding (the directory name is not a
    Python identifier, so it is loaded by path)."""
    spec = importlib.util.spec_from_file_location("lmx", os.path.join(PKG, "lmx.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def lmx():
    return load_lmx()


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    torch.cuda.init()
    return torch


@pytest.fixture
def mma_threshold(lmx):
    """Set the tensor-core threshold (smallest M routed to the tcgen05 path;
    0 = never) on the library and the oracle alike; restores the default."""
    import oracle_lib as O

    def set_(m):
        lmx.call("lmx_set_mma_min_m", m)
        O.lib().orc_set_mma_min_m(m)

    yield set_
    set_(16)
