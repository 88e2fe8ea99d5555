import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libtt_b200.so")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def tt_lib():
    """libtt_b200.so, built in-tree if it is missing (nvcc cross-compiles without a GPU)."""
    from tiktoktechjam2026_b200 import _lib
    from tiktoktechjam2026_b200.build import build

    if not os.path.exists(_lib.LIB_PATH):
        build()
    return _lib.lib()


@pytest.fixture(scope="session")
def golden():
    import json

    import numpy as np

    here = os.path.join(ROOT, "tests", "golden")
    data = np.load(os.path.join(here, "golden.npz"))
    with open(os.path.join(here, "golden_meta.json")) as f:
        meta = json.load(f)
    return data, meta


@pytest.fixture
def strict_fp32():
    import torch

    prev = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32,
            torch.get_float32_matmul_precision())
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev[0], prev[1]
    torch.set_float32_matmul_precision(prev[2])
