"""Shared test setup.

* ``gpu``-marked tests need a B200 (sm_100a) and the built ``libpi0b200.so``; everything else
  runs on CPU (oracle checks against the reference's golden outputs, host helpers, parameter
  table, C-ABI symbol exports).
* The drop-in package lives in ``mlc-vla_b200/`` and imports as ``mlc_vla`` (the reference's
  package name); the oracle (test infrastructure) imports as ``oracle``.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "mlc-vla_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built libpi0b200.so")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


def cosine(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-12))


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))
