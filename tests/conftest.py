import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); parity tests through the C ABI")
    config.addinivalue_line("markers", "slow: takes minutes (the oracle's side of a large config); still a gpu test")


@pytest.fixture(scope="session")
def tiny_model_path():
    from frizzle_b200 import synth
    return synth.model_path(synth.TINY, 0)


@pytest.fixture(scope="session")
def gemma_model_path():
    from frizzle_b200 import synth
    return synth.model_path(synth.GEMMA3_1B, 0)


@pytest.fixture(scope="session")
def device():
    from frizzle_b200.engine import Device
    d = Device(0)
    yield d
    d.close()


def rel_rms(got, want):
    import numpy as np
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.sqrt(np.mean((got - want) ** 2)) / max(np.sqrt(np.mean(want ** 2)), 1e-30))


def max_abs(got, want):
    import numpy as np
    return float(np.max(np.abs(np.asarray(got, dtype=np.float64) - np.asarray(want, dtype=np.float64))))
