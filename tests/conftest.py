"""pytest configuration: the `gpu` marker and shared fixtures.

Tests marked ``gpu`` need a CUDA device (they run on a B200 through the C ABI);
they are skipped, not passed, when no device is present.  Everything else runs
on the CPU.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def _cuda_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _cuda_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir():
    return os.path.join(ROOT, "tests", "golden")


@pytest.fixture(scope="session", autouse=True)
def _build_native():
    """Builds the in-tree CUDA library and the C oracle once per session (no-op when fresh)."""
    from aexrt_b200 import build

    build.build()
    import subprocess

    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle")], check=False,
                   stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
