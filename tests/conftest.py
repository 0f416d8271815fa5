import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG_PARENT = REPO / "fast-reduction_b200"
for p in (str(PKG_PARENT), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200 / sm_100a)")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_sessionstart(session):
    # Keep the in-tree libfrx.so in step with the sources (a no-op when it is up to date).
    sys.path.insert(0, str(PKG_PARENT))
    import build as frx_build  # fast-reduction_b200/build.py

    try:
        frx_build.build()
    except Exception as exc:  # reported by the tests that need the library
        print(f"[conftest] libfrx build failed: {exc}", file=sys.stderr)
