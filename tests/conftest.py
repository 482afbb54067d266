"""Shared pytest setup: the ``gpu`` marker, import paths, and the package under test.

``-m "not gpu"`` runs on any host (oracle vs golden fixtures, host logic, the C ABI's
exports). ``-m gpu`` runs the parity tests proper on a B200; without CUDA they are skipped
at collection time (they never fall back to a CPU path).
"""

from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
TESTS = Path(__file__).resolve().parent
if str(TESTS) not in sys.path:
    sys.path.insert(0, str(TESTS))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); the parity tests proper")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device on this host")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def uocr():
    return importlib.import_module("unlimited-ocr-max_b200")


@pytest.fixture(scope="session")
def oracle():
    from oracle import moe_oracle

    moe_oracle.build()
    return moe_oracle
