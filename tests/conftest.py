import os
import sys
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs on the GPU box)")
    config.addinivalue_line("markers", "slow: full-size (7B-shaped) case, minutes of runtime")


@pytest.fixture(scope="session")
def tiny_yalm():
    """The seeded synthetic tiny checkpoint (benchmark config 1)."""
    from yalm_b200 import synth
    path = os.path.join(tempfile.gettempdir(), "yalm_tiny_seed0.yalm")
    return synth.write_yalm(path, synth.SHAPES["tiny"], seed=0)


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "tiny_golden.npz")))


def have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def gpu():
    if not have_gpu():
        pytest.fail("test marked gpu but no CUDA device is visible")
    from yalm_b200 import build
    build.build_engine()
    return 0
