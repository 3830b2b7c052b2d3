"""Shared test setup.

* registers the ``gpu`` marker (tests that need a B200 are marked with it;
  ``-m "not gpu"`` runs the CPU suite);
* puts the repository root (for ``oracle``) and the package tree
  ``topk-tarmac_b200`` (for ``tarmac_b200`` and the drop-in ``src.*``
  modules) on ``sys.path``;
* ``golden(name)`` loads a committed fixture from ``tests/golden``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / "topk-tarmac_b200"
for p in (str(REPO), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200, sm_100a); run with -m gpu")


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    return torch.device("cuda:0")
