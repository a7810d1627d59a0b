"""Shared pytest setup: the ``gpu`` marker and golden-fixture loaders."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = Path(__file__).resolve().parent / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_fusions():
    return dict(np.load(GOLDEN / "fusions.npz"))


@pytest.fixture(scope="session")
def golden_relayout():
    return dict(np.load(GOLDEN / "relayout.npz"))


@pytest.fixture(scope="session")
def golden_ulysses():
    return dict(np.load(GOLDEN / "ulysses_w2.npz"))
