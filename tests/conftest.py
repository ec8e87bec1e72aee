import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built librce_qmm.so")


@pytest.fixture(scope="session")
def oracle():
    import oracle as o

    o.lib()
    return o


@pytest.fixture(scope="session")
def golden():
    path = os.path.join(ROOT, "tests", "golden", "qmm_golden.npz")
    return dict(np.load(path, allow_pickle=False))


@pytest.fixture(scope="session")
def ctx():
    import torch

    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    import rce_b200

    return rce_b200.default_context(0)
