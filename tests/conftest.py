"""Shared test setup.

* registers the ``gpu`` marker (tests that need a B200; run with ``-m gpu``);
* imports the package (its directory name is not an identifier) as ``qb``;
* imports the CPU oracle (``oracle/oracle.py``) that device results are checked against.
"""

from __future__ import annotations

import importlib
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)
ORACLE_DIR = os.path.join(REPO, "oracle")
if ORACLE_DIR not in sys.path:
    sys.path.insert(0, ORACLE_DIR)

PKG_NAME = "quaternion-based-math-1_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


def load_pkg():
    return importlib.import_module(PKG_NAME)


def load_submodule(name: str):
    return importlib.import_module(f"{PKG_NAME}.{name}")


@pytest.fixture(scope="session")
def qb():
    return load_pkg()


@pytest.fixture(scope="session")
def oracle():
    import oracle as o  # noqa: WPS433  (oracle/oracle.py, test infrastructure)

    o.build_c_oracle()
    return o


@pytest.fixture(scope="session")
def golden():
    return np.load(os.path.join(REPO, "tests", "golden", "golden.npz"))


@pytest.fixture(scope="session")
def workloads():
    return load_submodule("workloads")


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    load_pkg()._lib.load()  # fails loudly if the library is missing
    return torch.device("cuda", 0)
