"""Test configuration: the `gpu` marker and import paths.

Tests marked `gpu` need a B200 (sm_100) and the built libb200ops.so; the
rest run on any CPU host.  The oracle package (repo root) and the product
package (triton-agent_b200/) are put on sys.path here.
"""

import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "triton-agent_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU and the built CUDA library")


def _have_gpu() -> bool:
    try:
        import torch

        return torch.cuda.is_available() and torch.cuda.get_device_capability()[0] >= 10
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _have_gpu():
        return
    # Selecting `-m gpu` on a host without a GPU is an error in the run
    # configuration, not something to skip silently.
    if config.getoption("-m") and "not gpu" not in config.getoption("-m") and "gpu" in config.getoption("-m"):
        return
    skip = pytest.mark.skip(reason="needs an sm_100 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return REPO / "tests" / "golden"


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    assert torch.cuda.is_available(), "gpu tests need CUDA"
    return torch.device("cuda", 0)
