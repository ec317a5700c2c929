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


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to bf16/f16 (nearest even) and return them as float32."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    td = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dtype]
    return t.to(td).to(torch.float32).numpy()


def random_voxels(n: int, box: int, seed: int, batch: bool = False) -> np.ndarray:
    """n distinct voxels drawn uniformly from [0, box)^3 (int32 [n,3] or [n,4] with b=0)."""
    rng = np.random.default_rng(seed)
    flat = rng.choice(box ** 3, size=n, replace=False)
    c = np.stack([flat // (box * box), (flat // box) % box, flat % box], 1).astype(np.int32)
    if batch:
        c = np.concatenate([np.zeros((n, 1), np.int32), c], 1)
    return c
