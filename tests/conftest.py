"""Shared test set-up: the `gpu` marker, import paths and the oracle binding."""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "int4-gemv_b200")
for p in (PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu on a B200)")


@pytest.fixture(scope="session")
def oracle():
    import oracle_py
    return oracle_py.Oracle()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    g = np.load(os.path.join(ROOT, "tests", "golden", "golden.npz"))
    cases = sorted({k.split("/")[0] for k in g.files})
    return {c: {k.split("/")[1]: g[k] for k in g.files if k.startswith(c + "/")} for c in cases}


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import b4gemv
    b4gemv.load()  # the library must load: no fallback
    return torch.device("cuda:0")
