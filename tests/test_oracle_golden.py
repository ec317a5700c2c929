"""Pin the CPU oracle against the reference's own torch restatements (golden fixtures)."""
import numpy as np
import pytest

import oracle
from conftest import max_rel


def _tap_major_from_ref(nbr_ref):
    """The torch restatement's [N,27] table with -1 -> the tap-major [27*N], sentinel N."""
    n = nbr_ref.shape[0]
    t = nbr_ref.copy()
    t[t < 0] = n
    return np.ascontiguousarray(t.T).reshape(-1)


def test_neighbor_table_matches_reference(golden):
    g = golden["submconv"]
    nbr = oracle.build_neighbor_table(g["coords"])
    assert np.array_equal(nbr, _tap_major_from_ref(g["nbr_ref"]))


@pytest.mark.parametrize("case", ["dups", "origin_corner", "dense3", "isolated", "single", "far"])
def test_neighbor_table_edge_cases(golden, case):
    g = golden["nbr"]
    c = g[f"{case}_coords"]
    nbr = oracle.build_neighbor_table(c)
    assert np.array_equal(nbr, _tap_major_from_ref(g[f"{case}_nbr"]))
    # 4-column coords with batch 0 give the same map
    c4 = np.concatenate([np.zeros((c.shape[0], 1), np.int32), c], 1)
    assert np.array_equal(oracle.build_neighbor_table(c4), nbr)


def test_neighbor_table_structural():
    # centre tap t=13 is the row itself (unique coords); a dense 3^3 block gives the
    # interior voxel all 27 taps; empty input gives an empty map.
    c = np.stack(np.meshgrid(np.arange(3), np.arange(3), np.arange(3), indexing="ij"), -1).reshape(-1, 3)
    nbr = oracle.build_neighbor_table(c).reshape(27, -1)
    assert np.array_equal(nbr[13], np.arange(27))
    centre = 13  # (1,1,1) is row 13 in this enumeration
    assert np.all(nbr[:, centre] != 27)
    assert oracle.build_neighbor_table(np.zeros((0, 3), np.int32)).size == 0


def test_key_packing():
    assert oracle.key(0, 1, 2, 3) == (1 << 40) | (2 << 20) | 3
    # negative coordinates wrap exactly like the (uint32) casts of src/sparse.cpp:25
    assert oracle.key(0, 0, 0, -1) == 0xFFFFFFFF
    assert oracle.key(0, -1, 0, 0) == (0xFFFFFFFF << 40) & 0xFFFFFFFFFFFFFFFF


def test_submconv_matches_reference(golden):
    g = golden["submconv"]
    nbr = oracle.build_neighbor_table(g["coords"])
    out = oracle.submconv(nbr, g["feats"], g["weight"], g["bias"])
    assert max_rel(out, g["conv_out"]) < 1e-5


def test_submconv_isolated_voxel():
    rng = np.random.default_rng(0)
    ci, co = 8, 4
    c = np.array([[5, 5, 5], [20, 20, 20]], np.int32)
    f = rng.standard_normal((2, ci)).astype(np.float32)
    w = rng.standard_normal((co, 27, ci)).astype(np.float32)
    b = rng.standard_normal(co).astype(np.float32)
    out = oracle.submconv(oracle.build_neighbor_table(c), f, w, b)
    ref = f.astype(np.float64) @ w[:, 13, :].T.astype(np.float64) + b
    assert np.allclose(out, ref, rtol=0, atol=1e-12)


def test_submconv_f32_mt_matches_f64(golden):
    g = golden["submconv"]
    nbr = oracle.build_neighbor_table(g["coords"])
    ref = oracle.submconv(nbr, g["feats"], g["weight"], g["bias"], silu=True)
    wt = oracle.weight_tap_major(g["weight"].reshape(g["weight"].shape[0], 27, -1))
    out = oracle.submconv_f32_mt(nbr, g["feats"], wt, g["bias"], silu=True, nthreads=3)
    assert max_rel(out, ref) < 1e-5


def test_subdivide_matches_reference(golden):
    g = golden["c2s"]
    child, gidx, mstart = oracle.subdivide(g["coords"], g["mask"])
    assert np.array_equal(child, g["new_coords"])
    assert np.array_equal(gidx, g["gather_octant"] + 8 * g["gather_parent"])
    assert mstart[-1] == child.shape[0]
    assert np.all(np.diff(mstart) == g["mask"].sum(1))


def test_subdivide_mask_from_logits(golden):
    g = golden["c2s"]
    logits = g["feats"].astype(np.float64) @ g["to_subdiv.weight"].T.astype(np.float64) \
        + g["to_subdiv.bias"]
    # decisions agree except where the fp32 logit sits within rounding of 0
    sure = np.abs(g["subdiv"]) > 1e-5
    assert np.array_equal((logits > 0)[sure], g["mask"].astype(bool)[sure])


def test_c2s_block_matches_reference(golden):
    g = golden["c2s"]
    w = {k: g[k] for k in g if "." in k}
    w["conv1.weight"] = w["conv1.weight"].reshape(w["conv1.weight"].shape[0], 27, -1)
    w["conv2.weight"] = w["conv2.weight"].reshape(w["conv2.weight"].shape[0], 27, -1)
    out, child, mask = oracle.c2s_block(g["coords"], g["feats"], w, cout=16, ext_mask=g["mask"])
    assert np.array_equal(child, g["new_coords"])
    assert max_rel(out, g["out"]) < 1e-5


def test_convnext_tail_matches_reference(golden):
    # the ConvNeXt tail after the conv (src/sparse.cpp:124-133), restated in numpy
    g = golden["submconv"]
    nbr = oracle.build_neighbor_table(g["coords"])
    h = oracle.submconv(nbr, g["feats"], g["weight"], g["bias"])
    h = oracle.layer_norm(h, g["norm.weight"], g["norm.bias"])
    h = h @ g["mlp.0.weight"].T.astype(np.float64) + g["mlp.0.bias"]
    h = oracle.silu(h)
    h = h @ g["mlp.2.weight"].T.astype(np.float64) + g["mlp.2.bias"]
    h = h + g["feats"]
    assert max_rel(h, g["block_out"]) < 1e-5


@pytest.mark.skipif(not oracle.ref_nbr_available(), reason="oracle/_ref not built (the reference is absent)")
def test_oracle_map_equals_the_reference_function(tb, golden):
    """The oracle's map against the reference's own build_neighbor_table (its std::unordered_map
    loop, src/sparse.cpp:21-39, compiled from the reference's source): golden cases, negative and
    aliasing coordinates, duplicates (the later row wins), and a 250K-voxel shell."""
    from trellis_cpp_b200 import synth
    rng = np.random.default_rng(9)
    cases = [golden["submconv"]["coords"]] + [golden["nbr"][k] for k in golden["nbr"] if k.endswith("_coords")]
    cases.append(rng.integers(-3, 4, (3000, 3)).astype(np.int32))                  # negatives, duplicates
    big = rng.integers(0, 1 << 21, (2000, 3)).astype(np.int32)                       # keys alias past 2^20
    cases.append(np.concatenate([big, big[:50] + np.array([1, 0, 0], np.int32)]))
    cases.append(synth.coords_for("c2"))
    for c in cases:
        assert np.array_equal(oracle.build_neighbor_table(c), oracle.ref_build_neighbor_table(c))
