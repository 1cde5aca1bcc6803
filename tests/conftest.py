"""Shared pytest setup: the `gpu` marker and import paths.

CPU tests (`-m "not gpu"`) cover the oracle against the reference's golden
vectors, the host-side logic and the C-ABI exports. `-m gpu` tests drive the
CUDA path through the C ABI and compare with the oracle.
"""
import importlib
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG_NAME = "rust-ts-tokio-inference-engine_b200"
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device (run with -m gpu)")


def package():
    """Import the product package (its directory name carries hyphens)."""
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def pkg():
    return package()


@pytest.fixture(scope="session")
def O():
    import oracle
    oracle.build()
    return oracle


def has_cuda() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
