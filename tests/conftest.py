"""Shared pytest configuration.

Markers:
    gpu   needs a CUDA device (sm_100a); parity tests proper, calling the kernels through the C ABI.

Everything unmarked runs on a CPU-only machine: the oracle against the reference's golden vectors and against the
reference's own compiled sources, the C ABI library's exports and host-side validation, and the multi-rank host
logic over gloo.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for _p in (REPO, Path(__file__).resolve().parent):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import Reference, reference_available

    if not reference_available():
        pytest.skip("reference sources were not compiled into oracle/_ref (reference tree absent at build time)")
    return Reference()


@pytest.fixture(scope="session")
def golden():
    """Loads a committed fixture from tests/golden by file stem."""

    def load(name: str) -> dict[str, np.ndarray]:
        with np.load(GOLDEN_DIR / f"{name}.npz") as data:
            return {k: data[k] for k in data.files}

    return load


@pytest.fixture(scope="session")
def cuda():
    """The CUDA device and the loaded kernel library; GPU tests fail (not skip) when the library is missing."""
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from cppinf_b200 import capi

    capi.load()
    return torch.device("cuda", 0)
