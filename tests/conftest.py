import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "strands-decider-web_b200")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    """Import the product package from its (hyphenated) directory as ``strands_decider_web_b200``."""
    name = "strands_decider_web_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def ctx(pkg):
    """One library context on cuda:0 for the whole GPU session."""
    c = pkg.Context(0)
    yield c
    c.close()
