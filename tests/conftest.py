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


def _source_tree_dirs(root: str) -> list[str]:
    """The ``packages/*/src`` directories of a reference source checkout."""
    pk = os.path.join(root, "packages")
    if not os.path.isdir(pk):
        return []
    return sorted(os.path.join(pk, d, "src") for d in os.listdir(pk) if os.path.isdir(os.path.join(pk, d, "src")))


def reference_path():
    """Where the unmodified reference package can be imported from (or None).

    Looked up in order: ``baseline/_ref`` (what ``baseline/install_reference.sh`` lays
    down), then a reference source checkout named by ``SAINT_LLM_REFERENCE`` (its
    ``packages/*/src`` directories go on ``sys.path``; nothing is installed)."""
    installed = os.path.join(ROOT, "baseline", "_ref")
    if os.path.isdir(os.path.join(installed, "saint_llm_core")):
        return installed
    src = os.environ.get("SAINT_LLM_REFERENCE")
    if src:
        dirs = _source_tree_dirs(src)
        if any(os.path.isdir(os.path.join(d, "saint_llm_core")) for d in dirs):
            for d in dirs:
                if d not in sys.path:
                    sys.path.append(d)
            return dirs[0]
    return None


@pytest.fixture(scope="session")
def ref_pkgs():
    p = reference_path()
    if p is None:
        pytest.skip("reference package not found (baseline/_ref or SAINT_LLM_REFERENCE)")
    if p not in sys.path:
        sys.path.append(p)
    return p


@pytest.fixture
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")
