import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    path = os.path.join(ROOT, "oracle", "liboracle.so")
    if not os.path.exists(path):
        import subprocess
        subprocess.run(["make", "-s", "-f", os.path.join(ROOT, "oracle", "Makefile")], check=True)
    return Oracle(path)


@pytest.fixture(scope="session")
def golden_topology():
    return np.load(os.path.join(GOLDEN, "topology.npz"))


@pytest.fixture(scope="session")
def golden_features():
    return np.load(os.path.join(GOLDEN, "features.npz"))


@pytest.fixture(scope="session")
def ex():
    """The sm_100a executor; GPU tests fail (not skip) when it cannot be made."""
    import torch
    from mogecpp_b200.sparse import SparseCudaExecutor
    assert torch.cuda.is_available(), "GPU test run without a GPU"
    return SparseCudaExecutor(0)


def rel_l2(a, b):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, dtype=np.float64) - np.asarray(b, dtype=np.float64)))) if np.size(a) else 0.0
