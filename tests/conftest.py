import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "lisp-embed_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

SYNTH_ROOT = os.environ.get("EC_SYNTH_DIR", "/tmp/ec_synth")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def synth_root():
    os.makedirs(SYNTH_ROOT, exist_ok=True)
    return SYNTH_ROOT


@pytest.fixture(scope="session")
def ec():
    """The library, initialised on device 0 (GPU tests only)."""
    if not gpu_available():
        pytest.skip("no GPU")
    from embedcuda import _lib
    _lib.init([0])
    return _lib
