"""Shared test set-up: import paths, the `gpu` marker, CUDA fixtures."""

from __future__ import annotations

import sys
import warnings
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "ml-reentry-mlir_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = Path(__file__).resolve().parent / "golden"

warnings.filterwarnings("ignore", message=r".*Sparse CSR tensor support is in beta.*")


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a B200 (CUDA) device and the built libgnnc_b200.so"
    )
    config.addinivalue_line("filterwarnings", "ignore:.*Sparse CSR tensor support is in beta.*")


@pytest.fixture(scope="session")
def device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    # The product path must not fall back: a missing library is an error here.
    from gnnc.b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)
