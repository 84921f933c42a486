import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built sm_100a extension")
    config.addinivalue_line("markers", "slow: long-running test")
    config.addinivalue_line("markers", "distributed: spawns multiple processes")


def reference_path():
    """Where the unmodified reference package can be imported from (or None)."""
    cand = [os.path.join(ROOT, "baseline", "_ref")]
    for c in cand:
        if os.path.isdir(os.path.join(c, "saint_llm_core")):
            return c
    return None


@pytest.fixture(scope="session")
def ref_pkgs():
    p = reference_path()
    if p is None:
        pytest.skip("reference package not installed (baseline/_ref)")
    if p not in sys.path:
        sys.path.append(p)
    return p


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")
