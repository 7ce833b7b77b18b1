import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "qwen3.c_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, PKG_DIR)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_pkg():
    """Import the qwen3.c_b200 package (its directory name is not an identifier)."""
    if "qwen3c_b200" in sys.modules:
        return sys.modules["qwen3c_b200"]
    spec = importlib.util.spec_from_file_location(
        "qwen3c_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["qwen3c_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def golden(name):
    import numpy as np
    return np.load(os.path.join(ROOT, "tests", "golden", name))
