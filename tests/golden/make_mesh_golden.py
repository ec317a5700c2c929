#!/usr/bin/env python3
"""Generate ``mesh_ref.npz`` from the reference's own ``trellis::dual_grid_to_mesh``.

``src/dual_grid.cpp`` of the reference needs only the C++ standard library, so
``make -C oracle ref REF=<reference project>`` compiles it from its sources into
``oracle/_ref/libref_dual_grid.so`` (behind the C entry point of ``oracle/ref_dual_grid.cpp``).
This script runs that library on seeded cases and commits inputs and outputs; the tests then
pin the C restatement ``orc_dual_grid_mesh`` to them, and the GPU tests compare
``tb_dual_grid_mesh`` with both. The GPU box never runs this script.

Cases (key prefix ``<case>_``: coords [N,3] int32, f7 [N,7] float32, res, verts, faces):

* ``shell``: a seeded noisy spherical shell at res 32 (thickness 2), logits N(0, 2^2).
* ``dups``: the shell's first 200 voxels appended again with other fields (a later
  duplicate coordinate wins every lookup).
* ``special``: NaN intersected and split logits, split logits above 20 (softplus is the
  identity there), a block with every split logit 0 (equal products: always the 1-3
  diagonal), and voxels at coordinate 0.
* ``negative``: the shell shifted by -16 on every axis (negative coordinates, which alias
  under the packed key exactly as the reference's map treats them).
* ``one``: a single voxel (no quad can close).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle  # noqa: E402


def shell(res: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    g = np.arange(res)
    x, y, z = np.meshgrid(g, g, g, indexing="ij")
    r = np.sqrt((x - res / 2 + 0.5) ** 2 + (y - res / 2 + 0.5) ** 2 + (z - res / 2 + 0.5) ** 2)
    rad = res * 0.35 + rng.standard_normal() * 0.5
    keep = (np.abs(r - rad) < 1.0) & (rng.random(r.shape) < 0.97)
    return np.stack([x[keep], y[keep], z[keep]], 1).astype(np.int32)


def cases() -> dict:
    rng = np.random.default_rng(11)
    out = {}
    c = shell(32, 1)
    out["shell"] = (c, (rng.standard_normal((len(c), 7)) * 2).astype(np.float32), 32)
    cd = np.concatenate([c, c[:200]])
    out["dups"] = (cd, (rng.standard_normal((len(cd), 7)) * 2).astype(np.float32), 32)
    # special values on a dense 6^3 block at the origin
    g = np.arange(6)
    b = np.stack(np.meshgrid(g, g, g, indexing="ij"), -1).reshape(-1, 3).astype(np.int32)
    f = rng.standard_normal((len(b), 7)).astype(np.float32)
    f[::7, 3] = np.nan
    f[1::11, 4] = np.nan
    f[2::13, 6] = np.nan
    f[3::5, 6] = 25.0 + rng.random(len(f[3::5])).astype(np.float32)
    f[b[:, 0] >= 4, 6] = 0.0
    out["special"] = (b, f, 8)
    out["negative"] = (c - 16, (rng.standard_normal((len(c), 7)) * 2).astype(np.float32), 32)
    out["one"] = (np.array([[3, 4, 5]], np.int32), np.ones((1, 7), np.float32), 16)
    return out


def main():
    if not oracle.ref_available():
        sys.exit("build the reference library first: make -C oracle ref REF=<reference project>")
    arrays = {}
    for name, (c, f7, res) in cases().items():
        verts, faces = oracle.ref_dual_grid_mesh(c, f7, res)
        arrays.update({f"{name}_coords": c, f"{name}_f7": f7, f"{name}_res": np.int32(res),
                       f"{name}_verts": verts, f"{name}_faces": faces})
        print(f"{name}: N={len(c)} F={len(faces)}")
    np.savez_compressed(os.path.join(HERE, "mesh_ref.npz"), **arrays)


if __name__ == "__main__":
    main()
