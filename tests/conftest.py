"""Shared fixtures.  GPU tests are marked ``gpu``; everything else runs on CPU.

The product package is imported by its directory name.  The CPU oracle is
test infrastructure and is imported from ``oracle/`` only here.
"""
from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

PKG_NAME = "nemotron-webgpu-decode_b200"
GOLDEN = os.path.join(REPO, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: long-running")


def pytest_collection_modifyitems(config, items):
    # GPU tests on a machine without CUDA are skipped (the CPU suite runs with
    # -m "not gpu"); on a GPU machine a missing library fails loudly instead.
    try:
        import torch
        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def nwd():
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def ops(nwd):
    return importlib.import_module(PKG_NAME + ".ops")


@pytest.fixture(scope="session")
def engine_mod(nwd):
    return importlib.import_module(PKG_NAME + ".engine")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def golden():
    return np.load(GOLDEN)
