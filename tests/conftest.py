import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: long-running CPU test")


import pytest  # noqa: E402


@pytest.fixture(scope="session")
def gpu_backend():
    """A backend on cuda:0 that enqueues on torch's current stream."""
    import torch

    import openasr_b200 as ob

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but no CUDA device is visible")
    torch.cuda.init()
    be = ob.Backend(0)
    be.set_stream(torch.cuda.current_stream())
    yield be
    be.close()


def max_abs_rel(got, ref):
    import numpy as np

    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = np.abs(ref).max()
    return float(np.abs(got - ref).max() / (den if den > 0 else 1.0))
