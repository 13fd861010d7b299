import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(os.path.join(ROOT, "tests", "golden", "golden.npz")))


@pytest.fixture(scope="session")
def coracle():
    from oracle import oracle as O
    O.build()
    return O.COracle()


@pytest.fixture(scope="module")
def backend():
    """A CUDA backend on device 0.  Fails (does not skip) when the library or the GPU is
    missing: GPU tests must run the native path or fail."""
    from open_rknpu2_lm_infer_b200 import Backend
    b = Backend(device=0)
    yield b
    b.close()
