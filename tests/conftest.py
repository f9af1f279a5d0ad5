"""Shared test setup.

Markers: ``gpu`` -- needs a CUDA device (B200); everything else runs on CPU.
The oracle (oracle/) is imported here only as the checker.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "slow: long-running parity case")


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    return oracle


@pytest.fixture(scope="session")
def restated(oracle_mod):
    return oracle_mod.CEngine.restatement()


@pytest.fixture(scope="session")
def reference_engine(oracle_mod):
    eng = oracle_mod.CEngine.reference()
    if eng is None:
        pytest.skip("reference C engine not built here (oracle/_ref missing)")
    return eng


@pytest.fixture(scope="session")
def cuda_lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from gsdlq_b200 import _lib
    return _lib.load()


@pytest.fixture
def rng():
    return np.random.default_rng(1234)
