"""tb_dual_grid_mesh (trellis::dual_grid_to_mesh, src/dual_grid.cpp:16-56) on the GPU against the
reference's own outputs (tests/golden/mesh_ref.npz, written by the compiled reference) and the
oracle restatement pinned to them.

Tolerances: vertices within 1e-6 absolute (CUDA's expf and the host library's differ by at most
a couple of ulp; a vertex is about 0.5 in magnitude, ulp 6e-8). Triangle count and every quad's
corners exact; a quad's split may differ only where its two diagonal weight products are within
1e-5 relative of each other (log1pf/expf rounding), and then it must be the other split."""
import os
import shutil
import subprocess

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, ROOT

pytestmark = pytest.mark.gpu

CASES = ["shell", "dups", "special", "negative", "one"]


@pytest.fixture(scope="module")
def mesh_golden():
    return dict(np.load(os.path.join(GOLDEN, "mesh_ref.npz")))


def _case(g, name):
    return {k[len(name) + 1:]: v for k, v in g.items() if k.startswith(name + "_")}


def _other_split(q):
    """The same quad's two triangles split along the other diagonal."""
    if q[3] == q[0] and q[4] == q[2]:           # {q0,q1,q2, q0,q2,q3}
        q0, q1, q2, q3 = q[0], q[1], q[2], q[5]
        return np.array([q0, q1, q3, q3, q1, q2])
    q0, q1, q3, q2 = q[0], q[1], q[2], q[5]     # {q0,q1,q3, q3,q1,q2}
    return np.array([q0, q1, q2, q0, q2, q3])


def check_mesh(verts, faces, ref_verts, ref_faces, gap):
    assert verts.shape == ref_verts.shape
    nan = np.isnan(ref_verts)
    assert np.array_equal(np.isnan(verts), nan)
    if (~nan).any():
        assert np.max(np.abs(verts[~nan] - ref_verts[~nan])) <= 1e-6
    assert faces.shape == ref_faces.shape
    q, rq = faces.reshape(-1, 6), ref_faces.reshape(-1, 6)
    diff = np.nonzero(np.any(q != rq, axis=1))[0]
    for k in diff:
        assert gap[k] < 1e-5, f"quad {k}: split differs with margin {gap[k]}"
        assert np.array_equal(q[k], _other_split(rq[k])), f"quad {k}: not the other split"
    return len(diff)


def _run(c, f7, res, **kw):
    from trellis_cpp_b200 import ops
    v, f = ops.dual_grid_mesh(torch.from_numpy(c).cuda(), torch.from_numpy(f7).cuda(), res, **kw)
    ops.check_device()
    return v.cpu().numpy(), f.cpu().numpy()


@pytest.mark.parametrize("case", CASES)
def test_mesh_matches_reference(tb, mesh_golden, case):
    g = _case(mesh_golden, case)
    res = int(g["res"])
    verts, faces = _run(g["coords"], g["f7"], res)
    _, _, gap = oracle.dual_grid_mesh(g["coords"], g["f7"], res)
    check_mesh(verts, faces, g["verts"], g["faces"], gap)


def test_mesh_batch_column(tb, mesh_golden):
    # (b=0, x, y, z) rows key exactly like (x, y, z): the same mesh
    g = _case(mesh_golden, "dups")
    c4 = np.concatenate([np.zeros((len(g["coords"]), 1), np.int32), g["coords"]], 1)
    v3, f3 = _run(g["coords"], g["f7"], 32)
    v4, f4 = _run(c4, g["f7"], 32)
    assert np.array_equal(v3, v4) and np.array_equal(f3, f4)


# dups -1: rows left in ascending coordinate order (the map's sorted layout); 0: shuffled; > 0:
# that many duplicate rows appended
@pytest.mark.parametrize("res,dups", [(96, 0), (160, 2000), (128, -1)])
def test_mesh_large_shell(tb, res, dups):
    rng = np.random.default_rng(res)
    g = np.arange(res)
    x, y, z = np.meshgrid(g, g, g, indexing="ij")
    r = np.sqrt((x - res / 2) ** 2 + (y - res / 2) ** 2 + (z - res / 2) ** 2)
    keep = np.abs(r - res * 0.4) < 1.0
    c = np.stack([x[keep], y[keep], z[keep]], 1).astype(np.int32)
    if dups == 0:
        c = c[rng.permutation(len(c))]
    elif dups > 0:
        c = np.concatenate([c, c[rng.integers(0, len(c), dups)]])
    f7 = (rng.standard_normal((len(c), 7)) * 2).astype(np.float32)
    verts, faces = _run(c, f7, res)
    rv, rf, gap = oracle.dual_grid_mesh(c, f7, res)
    assert len(rf) > len(c) // 2
    check_mesh(verts, faces, rv, rf, gap)


def test_mesh_max_faces_and_empty(tb, mesh_golden):
    from trellis_cpp_b200 import ops
    g = _case(mesh_golden, "shell")
    nf = len(g["faces"])
    _, faces = _run(g["coords"], g["f7"], 32, max_faces=nf)
    assert faces.shape == g["faces"].shape
    with pytest.raises(ops.TBError) as e:
        _run(g["coords"], g["f7"], 32, max_faces=nf - 2)
    assert "max_faces" in str(e.value)
    v, f = _run(np.zeros((0, 3), np.int32), np.zeros((0, 7), np.float32), 32)
    assert v.shape == (0, 3) and f.shape == (0, 3)
    with pytest.raises(ops.TBError):
        _run(g["coords"], g["f7"], 0)


PROGRAM = r"""
#include "trellis_sparse.hpp"
#include <cstdio>
#include <cstdlib>
#include <string>
#include <vector>

int main(int argc, char** argv) {
    const std::string dir = argv[1];
    const int n = std::atoi(argv[2]);
    trellis::ShapeOut so;
    so.res = std::atoi(argv[3]);
    std::vector<int> c((size_t)n * 3);
    so.feats7.resize((size_t)n * 7);
    FILE* f = std::fopen((dir + "/in.bin").c_str(), "rb");
    if (!f || std::fread(c.data(), 4, c.size(), f) != c.size() ||
        std::fread(so.feats7.data(), 4, so.feats7.size(), f) != so.feats7.size()) return 2;
    std::fclose(f);
    so.coords.resize(n);
    for (int i = 0; i < n; ++i) so.coords[i] = {c[3 * i], c[3 * i + 1], c[3 * i + 2]};
    try {
        trellis::Mesh m = trellis::dual_grid_to_mesh(so);
        FILE* o = std::fopen((dir + "/out.bin").c_str(), "wb");
        std::fwrite(m.verts.data(), 4, m.verts.size(), o);
        std::fwrite(m.faces.data(), 4, m.faces.size(), o);
        std::fclose(o);
        std::printf("%d %d\n", m.V(), m.F());
    } catch (const std::exception& e) {
        std::fprintf(stderr, "exception: %s\n", e.what());
        return 1;
    }
    return 0;
}
"""


def test_mesh_cxx_mirror(tb, mesh_golden, tmp_path):
    cxx = shutil.which("g++") or pytest.skip("g++ not found")
    from trellis_cpp_b200 import _lib
    g = _case(mesh_golden, "dups")
    n = len(g["coords"])
    with open(tmp_path / "in.bin", "wb") as f:
        f.write(g["coords"].tobytes())
        f.write(g["f7"].tobytes())
    (tmp_path / "mesh.cpp").write_text(PROGRAM)
    cuda = "/usr/local/cuda"
    libdir = os.path.dirname(_lib.LIB_PATH)
    b = subprocess.run([cxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), "-I", cuda + "/include",
                        str(tmp_path / "mesh.cpp"), "-o", str(tmp_path / "mesh"), "-L", libdir, "-ltb_sparse",
                        "-Wl,-rpath," + libdir, "-L", cuda + "/lib64", "-lcudart", "-Wl,-rpath," + cuda + "/lib64"],
                       capture_output=True, text=True)
    assert b.returncode == 0, b.stderr
    r = subprocess.run([str(tmp_path / "mesh"), str(tmp_path), str(n), "32"], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    nv, nf = map(int, r.stdout.split())
    out = np.fromfile(tmp_path / "out.bin", dtype=np.float32)
    verts = out[: 3 * nv].reshape(nv, 3)
    faces = out[3 * nv:].view(np.int32).reshape(nf, 3)
    _, _, gap = oracle.dual_grid_mesh(g["coords"], g["f7"], 32)
    check_mesh(verts, faces, g["verts"], g["faces"], gap)
