import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from __graft_entry__ import load_package  # noqa: E402

load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def root():
    return ROOT


@pytest.fixture(scope="session")
def shipped_path():
    return os.path.join(ROOT, "models", "v001_eng.czm")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def shipped_oracle(oracle_mod, shipped_path):
    return oracle_mod.load_model(shipped_path)


@pytest.fixture(scope="session")
def pyref():
    import numpy as np

    return np.load(os.path.join(ROOT, "tests", "golden", "pyref_vectors.npz"))
