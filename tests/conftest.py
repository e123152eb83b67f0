"""Shared fixtures.  GPU tests are marked `gpu`; everything else runs on CPU."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


def normwise_rel(y, ref) -> float:
    """max_i |y_i - ref_i| / max_i |ref_i| (the parity metric of the GEMV path)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.max(np.abs(ref))
    return float(np.max(np.abs(y - ref)) / (den if den > 0 else 1.0))


def elem_rel_floor(y, ref, floor_frac: float = 1e-3) -> float:
    """max_i |y_i - ref_i| / max(|ref_i|, floor_frac * max|ref|): per-element
    relative error with a floor (rows that cancel to near zero would make the
    plain per-element ratio meaningless)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    den = np.maximum(np.abs(ref), floor_frac * max(float(np.max(np.abs(ref))), 1e-300))
    return float(np.max(np.abs(y - ref) / den))


# Parity bar of the GEMV path: normwise relative error against the fp32
# reference result.
GEMV_RTOL = 1e-4


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def patterns():
    return np.load(os.path.join(GOLDEN, "patterns.npz"))


@pytest.fixture(scope="session")
def seeded():
    return np.load(os.path.join(GOLDEN, "seeded.npz"))


@pytest.fixture(scope="session")
def sp():
    import sapphire_b200
    return sapphire_b200


@pytest.fixture(scope="session")
def ctx(sp):
    c = sp.Context(num_threads=4)
    yield c
    c.close()
