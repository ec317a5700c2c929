"""The oracle's dual-grid mesh restatement (orc_dual_grid_mesh, src/dual_grid.cpp:16-56) pinned
to the reference's own dual_grid_to_mesh: bit-exact against the committed fixtures that the
compiled reference wrote (tests/golden/make_mesh_golden.py), and against the compiled reference
itself on fresh inputs where oracle/_ref was built."""
import os

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

CASES = ["shell", "dups", "special", "negative", "one"]


@pytest.fixture(scope="module")
def mesh_golden():
    return dict(np.load(os.path.join(GOLDEN, "mesh_ref.npz")))


@pytest.mark.parametrize("case", CASES)
def test_oracle_mesh_matches_reference_fixture(mesh_golden, case):
    g = {k[len(case) + 1:]: v for k, v in mesh_golden.items() if k.startswith(case + "_")}
    verts, faces, gap = oracle.dual_grid_mesh(g["coords"], g["f7"], int(g["res"]))
    assert np.array_equal(verts, g["verts"], equal_nan=True)
    assert np.array_equal(faces, g["faces"])
    assert gap.size == faces.shape[0] // 2


def test_oracle_mesh_structure(mesh_golden):
    # every quad is two triangles on present voxels, split along one diagonal
    c, f7 = mesh_golden["shell_coords"], mesh_golden["shell_f7"]
    verts, faces, _ = oracle.dual_grid_mesh(c, f7, 32)
    assert faces.shape[0] % 2 == 0 and faces.min() >= 0 and faces.max() < len(c)
    quads = faces.reshape(-1, 6)
    split1 = (quads[:, 3] == quads[:, 0]) & (quads[:, 4] == quads[:, 2])
    split2 = (quads[:, 2] == quads[:, 3]) & (quads[:, 4] == quads[:, 1])
    assert np.all(split1 ^ split2)
    # vertices lie within half a voxel outside their voxel's cell, inside the world cube
    lo = (c - 0.5) / 32 - 0.5
    assert np.all(verts >= lo - 1e-6) and np.all(verts <= lo + 2.0 / 32 + 1e-6)


def test_oracle_mesh_empty():
    verts, faces, gap = oracle.dual_grid_mesh(np.zeros((0, 3), np.int32), np.zeros((0, 7), np.float32), 8)
    assert verts.shape == (0, 3) and faces.shape == (0, 3) and gap.size == 0


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref not built (needs the reference sources)")
@pytest.mark.parametrize("seed", [0, 1])
def test_oracle_mesh_matches_reference_library(seed):
    rng = np.random.default_rng(seed)
    flat = rng.choice(40 ** 3, size=20000, replace=False)
    c = np.stack([flat // 1600, (flat // 40) % 40, flat % 40], 1).astype(np.int32)
    c = np.concatenate([c, c[rng.integers(0, len(c), 500)]])
    f7 = (rng.standard_normal((len(c), 7)) * 3).astype(np.float32)
    verts, faces, _ = oracle.dual_grid_mesh(c, f7, 40)
    rv, rf = oracle.ref_dual_grid_mesh(c, f7, 40)
    assert np.array_equal(verts, rv) and np.array_equal(faces, rf)
