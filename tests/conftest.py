"""pytest setup: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle-vs-golden checks, host logic and the C-ABI
load/export checks on CPU; `-m gpu` runs the parity tests on a B200.
"""
import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "vpipe-ltx-2.5_b200")
for p in (REPO, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers",
                            "gpu: needs an sm_100a GPU (B200); parity tests")


@pytest.fixture(scope="session")
def ctx():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import ltx25_b200 as L
    c = L.Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    d = os.path.join(REPO, "tests", "golden")

    def load(name):
        return np.load(os.path.join(d, name))
    return load
