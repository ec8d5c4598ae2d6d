import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "flint-vllm-single-dgx-spark_b200")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def load_package():
    """Import the product package (its directory name is not a Python identifier) as ``flint_b200``."""
    if "flint_b200" in sys.modules:
        return sys.modules["flint_b200"]
    spec = importlib.util.spec_from_file_location(
        "flint_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["flint_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def fb():
    return load_package()


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", "reference_golden.npz"))
