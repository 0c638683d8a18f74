"""Shared pytest set-up: the `gpu` marker, import paths, and config builders."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "sparse-matrix-multiplication_b200"
for p in (str(REPO), str(PKG), str(Path(__file__).resolve().parent)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def cuda():
    """torch with a usable CUDA device (GPU tests only)."""
    import torch

    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    torch.cuda.init()
    return torch
