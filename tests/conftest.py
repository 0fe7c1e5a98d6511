"""Shared pytest setup: the `gpu` marker, import paths and fixtures."""
import importlib.util
import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(REPO, "mlx-confucius4-tts_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
sys.path.insert(0, os.path.join(REPO, "oracle"))


def load_c4s():
    """Import the package directory `mlx-confucius4-tts_b200/` as module `c4s`."""
    if "c4s" in sys.modules:
        return sys.modules["c4s"]
    spec = importlib.util.spec_from_file_location(
        "c4s", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["c4s"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def c4s():
    return load_c4s()


@pytest.fixture(scope="session")
def oracle():
    import oracle as orc
    return orc.Oracle()


@pytest.fixture(scope="session")
def golden_proc():
    return dict(np.load(os.path.join(GOLDEN, "ref_proc.npz")))


@pytest.fixture(scope="session")
def golden_chain():
    return dict(np.load(os.path.join(GOLDEN, "ref_chain.npz")))
