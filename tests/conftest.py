"""Shared test setup: markers, import paths, the library and the oracle."""
import importlib
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

PKG_NAME = "15-618_dynamic_sparse_decode_b200"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_pkg():
    return importlib.import_module(PKG_NAME)


@pytest.fixture(scope="session")
def dsd():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as o
    o.lib()
    return o
