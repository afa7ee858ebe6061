import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "dist: multi-process (torch.distributed) test")


@pytest.fixture(scope="session")
def golden():
    def load(name):
        return np.load(os.path.join(GOLDEN, name), allow_pickle=False)

    return load


@pytest.fixture(scope="session")
def lib():
    """The product library (built in-tree if missing)."""
    from gguf_onnx_ops_b200 import build as b

    if not os.path.exists(b.LIB):
        b.build()
    from gguf_onnx_ops_b200 import _lib

    return _lib.load()


@pytest.fixture(scope="session")
def cuda(lib):
    import torch

    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    torch.cuda.init()
    return torch.device("cuda:0")
