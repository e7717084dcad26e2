"""Shared test setup: import paths, the ``gpu`` marker, fixtures."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "asterlm-frontier_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libasterq.so")


@pytest.fixture(scope="session")
def golden_encode():
    return dict(np.load(GOLDEN / "encode_golden.npz"))


@pytest.fixture(scope="session")
def golden_decode():
    return dict(np.load(GOLDEN / "decode_golden.npz"))


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test needs a CUDA device")
    from asterq import _lib

    _lib.load()
    return torch.device("cuda:0")
