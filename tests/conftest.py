"""Shared pytest setup: the `gpu` marker, package loading and fixture paths."""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def load_package():
    """Import the product package (its directory name has a dot, so load it by path)."""
    if "trellis_cpp_b200" in sys.modules:
        return sys.modules["trellis_cpp_b200"]
    pkg_dir = os.path.join(ROOT, "trellis.cpp_b200")
    spec = importlib.util.spec_from_file_location(
        "trellis_cpp_b200", os.path.join(pkg_dir, "__init__.py"),
        submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["trellis_cpp_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def tb():
    return load_package()


@pytest.fixture(scope="session")
def golden():
    return {
        "submconv": dict(np.load(os.path.join(GOLDEN, "submconv_ref.npz"))),
        "c2s": dict(np.load(os.path.join(GOLDEN, "c2s_ref.npz"))),
        "nbr": dict(np.load(os.path.join(GOLDEN, "nbr_cases.npz"))),
    }


def max_rel(mine, ref):
    """max|mine - ref| / max|ref|, the reference's metric (src/test_sparse_conv.cpp:16-23)."""
    mine = np.asarray(mine, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.max(np.abs(mine - ref)) / max(np.max(np.abs(ref)), 1e-30))
