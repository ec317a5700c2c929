"""GPU neighbor map vs the reference's semantics: bit-exact against the golden fixtures
(the reference's own torch restatement) and against the C oracle at full config sizes."""
import numpy as np
import pytest
import torch

import oracle
from conftest import random_voxels

pytestmark = pytest.mark.gpu


def _gpu_map(coords_np):
    from trellis_cpp_b200 import ops
    c = torch.from_numpy(np.ascontiguousarray(coords_np, dtype=np.int32)).cuda()
    nbr = ops.build_neighbor_table(c)
    ops.check_device()
    return nbr.cpu().numpy()


def _ref_tap_major(nbr_ref):
    t = nbr_ref.copy()
    t[t < 0] = nbr_ref.shape[0]
    return np.ascontiguousarray(t.T).reshape(-1)


def test_golden_submconv_map(tb, golden):
    g = golden["submconv"]
    assert np.array_equal(_gpu_map(g["coords"]), _ref_tap_major(g["nbr_ref"]))


@pytest.mark.parametrize("case", ["dups", "origin_corner", "dense3", "isolated", "single", "far"])
def test_golden_edge_cases(tb, golden, case):
    g = golden["nbr"]
    assert np.array_equal(_gpu_map(g[f"{case}_coords"]), _ref_tap_major(g[f"{case}_nbr"]))


def test_empty(tb):
    from trellis_cpp_b200 import ops
    out = ops.build_neighbor_table(torch.zeros((0, 3), dtype=torch.int32, device="cuda"))
    assert out.numel() == 0


def test_negative_special_and_aliasing_keys(tb):
    # (-1,-1,-1) packs to the all-ones key; coords >= 2^20 alias exactly as the reference's
    # 64-bit packing does; negative coords wrap through the uint32 casts.
    c = np.array([[-1, -1, -1], [0, 0, 0], [-1, 0, 0], [5, -3, 7], [1 << 20, 0, 0], [0, 1, 0],
                  [2, 2, 2], [-1, -1, -2], [(1 << 20) - 1, 3, 3], [0, 0, -1]], np.int32)
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


def test_random_duplicates(tb):
    rng = np.random.default_rng(7)
    c = rng.integers(0, 12, size=(5000, 3)).astype(np.int32)   # ~3x duplicated
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


def test_batch_column(tb):
    rng = np.random.default_rng(8)
    c = np.concatenate([rng.integers(0, 4, (4000, 1)), rng.integers(0, 10, (4000, 3))], 1).astype(np.int32)
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


def test_partial_tiles_and_sizes(tb):
    for n in (1, 2, 127, 128, 129, 1000, 4097):
        c = random_voxels(n, 24, n)
        assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c)), n


@pytest.mark.parametrize("name", ["c1", "c2", "c4", "c5_32"])
def test_config_maps_full_size(tb, name):
    from trellis_cpp_b200 import synth
    c = synth.coords_for(name)
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


# The map is built in 4x4x4 coordinate blocks when every coordinate is in [0, 2^20 - 2] and every
# batch index in [0, 15], with buckets for at most N/4 + 64 blocks; otherwise the voxel hash
# builds it. Both must give the reference's map; these cases sit on either side of each limit.
@pytest.mark.parametrize("top", [(1 << 20) - 2, (1 << 20) - 1])
def test_block_layout_coordinate_limit(tb, top):
    rng = np.random.default_rng(top & 0xFF)
    c = random_voxels(3000, 16, 31).astype(np.int64)
    c[:1000] = c[:1000] % 14 + (top - 13)       # a cluster reaching exactly the top of the range
    c[1000:1500, 0] = top - rng.integers(0, 3, 500)
    assert c.max() == top or c.max() < top
    c = np.concatenate([c, [[0, 0, 0], [top, top, top], [top, 0, top], [top - 1, top, top]]]).astype(np.int32)
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


@pytest.mark.parametrize("bmax", [15, 16])
def test_block_layout_batch_limit(tb, bmax):
    rng = np.random.default_rng(bmax)
    c = np.concatenate([rng.integers(0, bmax + 1, (6000, 1)), rng.integers(0, 9, (6000, 3))], 1).astype(np.int32)
    c[0, 0] = bmax
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


@pytest.mark.parametrize("spacing", [1, 4, 5])
def test_block_layout_sparse_overflow(tb, spacing):
    # spacing >= 4 puts every voxel in its own block: more blocks than buckets, so the voxel hash
    # builds the map (spacing 4 also makes every neighbor absent)
    g = np.stack(np.meshgrid(*[np.arange(0, 24 * spacing, spacing)] * 3, indexing="ij"), -1).reshape(-1, 3)
    rng = np.random.default_rng(spacing)
    c = g[rng.permutation(g.shape[0])].astype(np.int32)
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


def test_block_layout_shuffled_shell_with_duplicates(tb):
    from trellis_cpp_b200 import synth
    c = synth.coords_for("c2")
    rng = np.random.default_rng(4)
    c = np.concatenate([c, c[rng.integers(0, c.shape[0], 20000)]])
    c = c[rng.permutation(c.shape[0])]
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


@pytest.mark.skipif(not oracle.ref_nbr_available(), reason="oracle/_ref not built (the reference is absent)")
@pytest.mark.parametrize("name", ["c1", "c2"])
def test_gpu_map_equals_the_reference_function(tb, name):
    """The device map against the reference's own build_neighbor_table (src/sparse.cpp:21-39,
    compiled from its source into oracle/_ref), bit for bit."""
    from trellis_cpp_b200 import ops, synth
    c = synth.coords_for(name)
    got = ops.build_neighbor_table(torch.from_numpy(c).cuda()).cpu().numpy()
    assert np.array_equal(got, oracle.ref_build_neighbor_table(c))


def _big_cases():
    """Inputs of 300k voxels: duplicates (the later row wins), batches, voxels on every face of
    the bounding box, a negative coordinate (which sends the build to the voxel hash), and a
    bounding box of ~1e15 cells."""
    rng = np.random.default_rng(12)
    n = 300_000
    dup = rng.integers(0, 64, (n, 3)).astype(np.int32)                     # ~1.1x duplicated, box faces hit
    bat = np.concatenate([rng.integers(0, 5, (n, 1)), rng.integers(100, 160, (n, 3))], 1).astype(np.int32)
    far = random_voxels(n, 70, 13)
    far[::1000] += np.array([900_000, 0, 0], np.int32)                         # bounding box of ~1e15 cells
    bad = random_voxels(n, 70, 14)
    bad[5] = [-3, 4, 5]                                                       # negative: the voxel hash builds it
    return [("duplicates", dup), ("batches", bat), ("huge box", far), ("negative", bad)]


@pytest.mark.parametrize("case", ["duplicates", "batches", "huge box", "negative"])
def test_large_builds_all_layouts(tb, case):
    c = dict(_big_cases())[case]
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


def test_builds_in_a_row_are_independent(tb):
    """Builds in a row on different voxel sets of one context: each must match the oracle, so
    the buckets an earlier build wrote cannot leak into a later one."""
    from trellis_cpp_b200 import synth
    sets = [synth.coords_for("c5_32")[:400_000], random_voxels(280_000, 80, 15), synth.coords_for("c5_32")[::7]]
    for c in sets + sets[:1]:
        assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


# Rows in strictly ascending (batch, x, y, z) order build the map from a table of (batch, x, y)
# columns (the sorted layout); rows in any other order, repeated coordinates, coordinates outside
# [0, 2^20 - 2] or a bounding box with more columns than the table holds go to the block layout.
# These cases sit on either side of each condition and must all give the reference's map.
def _sorted(c):
    c = np.asarray(c, np.int64)
    k = (c[:, 0] << 60) | (c[:, 1] << 40) | (c[:, 2] << 20) | c[:, 3] if c.shape[1] == 4 else \
        (c[:, 0] << 40) | (c[:, 1] << 20) | c[:, 2]
    return c[np.argsort(k, kind="stable")].astype(np.int32)


def _sorted_cases():
    rng = np.random.default_rng(21)
    dup_col = np.concatenate([rng.integers(0, 3, (4000, 1)), rng.integers(0, 9, (4000, 3))], 1)
    dup_col[:1500] = [1, 4, 4, 5]                        # one voxel 1500 times: the binary-search path
    long_cols = np.concatenate([np.zeros((6000, 1), np.int64), rng.integers(0, 2, (6000, 2)),
                                rng.integers(0, 4000, (6000, 1))], 1)       # 4 columns of ~1500 rows
    long_cols = np.unique(long_cols, axis=0)                                  # distinct: the sorted layout
    top = (1 << 20) - 2
    edges = np.array([[0, 0, 0, 0], [0, 0, 0, 1], [0, 0, 1, 0], [0, 1, 0, 0], [0, top, top, top],
                      [0, top - 1, top, top], [0, top, top - 1, top], [0, top, top, top - 1],
                      [15, 0, 0, 0], [15, 0, 0, 1]])                      # 2^40 columns: block layout
    small_box = np.concatenate([rng.integers(0, 16, (3000, 1)), rng.integers(0, 6, (3000, 3))], 1)
    return {"duplicates": _sorted(dup_col), "long columns": _sorted(long_cols),
            "huge box": _sorted(edges), "batches 0-15": _sorted(small_box),
            "3-column coords": _sorted(random_voxels(5000, 20, 22))}


@pytest.mark.parametrize("case", ["duplicates", "long columns", "huge box", "batches 0-15", "3-column coords"])
def test_sorted_layout(tb, case):
    c = _sorted_cases()[case]
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


@pytest.mark.parametrize("change", ["one pair swapped", "negative coordinate", "batch 16", "last row first"])
def test_sorted_layout_rejections(tb, change):
    from trellis_cpp_b200 import synth
    c = synth.coords_for("c2").copy()
    if change == "one pair swapped":
        c[[1000, 1001]] = c[[1001, 1000]]
    elif change == "negative coordinate":
        c[0, 1] = -1
    elif change == "batch 16":
        c[-1, 0] = 16
    else:
        c = np.concatenate([c[-1:], c[:-1]])
    assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))


def test_sorted_and_unsorted_builds_alternate(tb):
    """The sorted layout's column table and the block layout's buckets share memory: builds that
    alternate between the layouts on one context must each match the oracle."""
    from trellis_cpp_b200 import synth
    s = synth.coords_for("c2")
    u = s[np.random.default_rng(23).permutation(s.shape[0])]
    for c in (s, u, s, u[:7000], s[:9000]):
        assert np.array_equal(_gpu_map(c), oracle.build_neighbor_table(c))

