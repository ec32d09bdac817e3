"""Shared pytest setup: the ``gpu`` marker and import paths."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


def cuda_available() -> bool:
    import torch

    return torch.cuda.is_available()


@pytest.fixture(scope="session")
def golden_dir() -> Path:
    return REPO / "tests" / "golden"


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def tol(ref) -> float:
    """The north star's error bound: max-abs error <= 2e-2 relative to the fp32
    reference's scale, i.e. 2e-2 * max(1, max|ref|)."""
    return 2e-2 * max(1.0, float(ref.abs().max()))
