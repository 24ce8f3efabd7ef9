"""Shared pytest setup.

Markers: `gpu` tests need a B200 and the built sm_100a library; everything
else runs on CPU.  The oracle (oracle/) is test infrastructure and is
imported only here and in tests.
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "llm-inference-diy_b200")
ORACLE = os.path.join(ROOT, "oracle")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (PKG, ORACLE, GOLDEN):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built sm_100a library")


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc_mod
    return orc_mod.Oracle()


@pytest.fixture(scope="session")
def rng():
    import numpy as np
    return np.random.default_rng(1234)


def cuda_available() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
