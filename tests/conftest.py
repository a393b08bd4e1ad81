import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size workload")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    path = os.path.join(ROOT, "tests", "golden", "golden.npz")
    with np.load(path) as z:
        return {k: z[k] for k in z.files}


def gen(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


@pytest.fixture(scope="session")
def golden_moe():
    """Outputs of the reference's NaiveMoEMLP (tests/golden/make_moe_golden.py)."""
    import numpy as np
    path = os.path.join(ROOT, "tests", "golden", "golden_moe.npz")
    with np.load(path) as z:
        return {k: z[k] for k in z.files}
