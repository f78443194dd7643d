"""Shared fixtures.  Tests marked ``gpu`` need a CUDA device (B200); the rest
run on any CPU host and must not launch GPU work."""
from __future__ import annotations

import importlib.util
import os
import sys

import pytest

ROOT = os.path.abspath(os.path.join(os.path.dirname(__file__), ".."))
PKG_DIR = os.path.join(ROOT, "tmac_gguf.cpp_b200")
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests", "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)


def load_package():
    """Import the package directory (its name contains a dot, so it is
    loaded by path under the module name tmac_gguf_cpp_b200)."""
    name = "tmac_gguf_cpp_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(
        name, os.path.join(PKG_DIR, "__init__.py"),
        submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


@pytest.fixture(scope="session")
def tg():
    return load_package()


@pytest.fixture(scope="session")
def O():
    import oracle
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cases():
    import cases as c
    return c


@pytest.fixture(scope="module")
def backend(tg):
    b = tg.CudaBackend(0)
    yield b
    b.shutdown()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_ref.npz"))


@pytest.fixture(scope="session")
def golden_qkv():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "golden_qkv.npz"))
