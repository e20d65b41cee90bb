"""Shared fixtures.  `-m gpu` tests need a B200 and the built runtime library;
everything else runs on CPU (oracle vs golden vectors, host logic, ABI load)."""
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU and libmalus_runtime_cuda.so")


@pytest.fixture(scope="session")
def orc():
    from oracle import pyoracle
    pyoracle.build()
    pyoracle.load()
    return pyoracle


@pytest.fixture(scope="session")
def rt():
    import malus_b200
    lib = malus_b200.load()
    return lib


@pytest.fixture(scope="session")
def M():
    import malus_b200
    malus_b200.load()
    return malus_b200


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def rel_err(got, ref, scale=None):
    """max |got-ref| / max(scale or |ref|, tiny) — scale lets callers normalise
    by sum|terms| as the matmul/reduction tolerances prescribe."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if scale is None:
        scale = np.abs(ref)
    scale = np.maximum(np.asarray(scale, np.float64), 1e-30)
    return float(np.max(np.abs(got - ref) / scale)) if got.size else 0.0
