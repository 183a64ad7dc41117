"""Shared test setup.

Markers: `gpu` = needs a B200 (run with -m gpu); everything else runs on CPU.
Paths: the package binding (mxfp6-gemm_b200/mxfp6_b200) and the CPU oracle (oracle/) are put
on sys.path here; the oracle is only ever the checker.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "mxfp6-gemm_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def oracle():
    from oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def lib():
    import mxfp6_b200
    return mxfp6_b200
