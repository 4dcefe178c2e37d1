"""Shared test setup.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``);
* puts the package root (``clifford-space-network_b200/``, which holds ``csn_b200``
  and the reference-compatible ``python`` / ``csn`` packages) and the repository
  root (for ``oracle``) on ``sys.path``.
"""
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
PKG_ROOT = REPO / "clifford-space-network_b200"
for p in (str(PKG_ROOT), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        with np.load(GOLDEN / f"{name}.npz") as f:
            return {k: f[k] for k in f.files}
    return load


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as orc
    orc.build()
    return orc
