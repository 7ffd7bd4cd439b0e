"""Shared pytest setup: the `gpu` marker, the package loader and the oracle path."""
from __future__ import annotations

import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "penumbra-fhe_b200")
ORACLE_DIR = os.path.join(ROOT, "oracle")
GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")

if ORACLE_DIR not in sys.path:
    sys.path.insert(0, ORACLE_DIR)


def load_package():
    """Import the package directory ``penumbra-fhe_b200`` as module ``penumbra_b200``."""
    if "penumbra_b200" in sys.modules:
        return sys.modules["penumbra_b200"]
    spec = importlib.util.spec_from_file_location(
        "penumbra_b200", os.path.join(PKG_DIR, "__init__.py"),
        submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["penumbra_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def pnb():
    return load_package()


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.lib()
    return O
