"""Shared fixtures.  Marker `gpu`: needs a B200 (run with -m gpu)."""
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "42-berlin-engine_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))


def load_pkg_module(name):
    """Import a module from the package directory (its name is not a valid
    Python identifier, so it is loaded by path)."""
    key = "ec_" + name
    if key in sys.modules:
        return sys.modules[key]
    spec = importlib.util.spec_from_file_location(key, os.path.join(PKG, name + ".py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[key] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def synth():
    return load_pkg_module("synth")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    if not os.path.exists(O.PORT_SO):
        pytest.skip("oracle/libec_port.so not built (run __graft_entry__.build())")
    return O


@pytest.fixture(scope="session")
def ref(oracle):
    if not oracle.ref_available():
        pytest.skip("reference oracle oracle/_ref not built here")
    return oracle


@pytest.fixture(scope="session")
def tiny_model(synth):
    return synth.make_model(synth.TINY, seed=7)
