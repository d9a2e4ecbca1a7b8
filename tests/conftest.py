"""Shared pytest setup: import paths, the ``gpu`` marker, common fixtures."""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "cortex-engine_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="CUDA device required")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden_kernels():
    return torch.load(os.path.join(GOLDEN, "golden_kernels.pt"), weights_only=False)


@pytest.fixture(scope="session")
def golden_models():
    return torch.load(os.path.join(GOLDEN, "golden_models.pt"), weights_only=False)


@pytest.fixture(scope="session")
def golden_ingest():
    return torch.load(os.path.join(GOLDEN, "golden_ingest.pt"), weights_only=False)
