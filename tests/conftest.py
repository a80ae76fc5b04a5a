"""Test configuration: markers, package/oracle loading, shared fixtures.

`-m gpu` tests need a B200 and call the C ABI of libg4b200.so; everything else
runs on the CPU (oracle pinning, golden fixtures, host logic, ABI exports).
"""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "gemma4.c_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def load_pkg():
    if "g4b200" in sys.modules:
        return sys.modules["g4b200"]
    spec = importlib.util.spec_from_file_location("g4b200", os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["g4b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


@pytest.fixture(scope="session")
def g4():
    return load_pkg()


@pytest.fixture(scope="session")
def orc():
    import oracle
    return oracle.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle
    if not oracle.have_reference():
        pytest.skip("reference build oracle/_ref/libg4ref.so absent")
    return oracle.Reference()


@pytest.fixture(scope="session")
def ref_generic():
    """The reference built with -DGEMMA4_USE_GENERIC_DOT (its scalar dot kernels): the spread
    between the two reference builds is the reference's own float noise."""
    import oracle
    path = oracle.REF_SO.replace("libg4ref.so", "libg4ref_generic.so")
    if not os.path.exists(path):
        pytest.skip("generic reference build absent")
    return oracle.Reference(path=path)


@pytest.fixture(scope="session")
def golden():
    path = os.path.join(ROOT, "tests", "golden", "golden.npz")
    return dict(np.load(path, allow_pickle=False))


@pytest.fixture
def gpu(g4):
    """The per-call API with a clean weight registry (fails loudly when the
    library is missing; skips only when the machine has no CUDA device)."""
    L = g4.lib()
    rc = L.g4_set_device(0)
    if rc == g4.G4_ERR_NO_DEVICE:
        pytest.skip("no CUDA device: " + g4.last_error()[1])
    assert rc == 0, g4.last_error()
    g4.registry_clear()
    yield g4
    g4.registry_clear()
