import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (runs the CUDA bridge)")


@pytest.fixture(scope="session")
def bridge_lib():
    """Builds (if stale) and loads libcudabridge.so."""
    from rustane_b200 import build, bridge
    build.build()
    return bridge.load_library()


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    oracle.build()
    return oracle.lib()


def pytest_collection_modifyitems(config, items):
    """GPU tests need a visible CUDA device; without one they are skipped."""
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)
