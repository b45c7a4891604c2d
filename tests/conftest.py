"""Shared test setup: the ``gpu`` marker, the package import under its alias, and the library build.

CPU tests (``-m "not gpu"``) cover the oracle against the reference's golden vectors, the host-side logic and the
C-ABI library's exports; ``-m gpu`` tests call the CUDA kernels through the C ABI and compare with the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def zb():
    """The package, with its C-ABI library built (nvcc cross-compiles when it is missing or stale)."""
    lib = __graft_entry__.PACKAGE_DIR / "libzonos3_b200.so"
    if not lib.exists():
        __graft_entry__.build()
    pkg = __graft_entry__.load_package()
    pkg._lib.load()
    return pkg


@pytest.fixture(scope="session")
def golden():
    def load(name):
        with np.load(GOLDEN / name) as f:
            return {k: torch.from_numpy(f[k].copy()) for k in f.files}

    return load


def rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """||a - b|| / ||b|| in float64."""
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def max_rel_err(a: torch.Tensor, b: torch.Tensor) -> float:
    """max |a - b| / max |b| in float64."""
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()
