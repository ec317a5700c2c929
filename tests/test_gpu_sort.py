"""tb_sort_rows: the stable key-order permutation the decoder's stages use for their map and
ConvNeXt blocks. The order is the reference's voxel key (b, x, y, z), src/sparse.cpp:25, so the
expected permutation is numpy's stable lexsort of the same columns; integer data, checked exactly."""
import numpy as np
import pytest
import torch

from conftest import random_voxels

pytestmark = pytest.mark.gpu


def _expected(coords):
    cols = [coords[:, k] for k in range(coords.shape[1] - 1, -1, -1)]     # last key column first
    return np.lexsort(cols, axis=0).astype(np.int32)


def _cases():
    from trellis_cpp_b200 import synth
    rng = np.random.default_rng(5)
    dups = rng.integers(-3, 9, size=(5000, 3)).astype(np.int32)          # repeats and negatives
    batch = np.concatenate([rng.integers(0, 3, (4000, 1)), rng.integers(0, 40, (4000, 3))], axis=1).astype(np.int32)
    shell = synth.coords_for("c2")                                        # [N,4], already in key order
    # parent-major children of a shuffled parent set (the order the C2S block returns)
    par = random_voxels(3000, 64, 9)[rng.permutation(3000)]
    child = (2 * par[:, None, :] + np.array([[o & 1, (o >> 1) & 1, o >> 2] for o in range(8)], np.int32)[None]).reshape(-1, 3)
    return [("duplicates and negatives", dups), ("batch column", batch), ("sorted shell", shell),
            ("parent-major children", child), ("one row", np.array([[7, 8, 9]], np.int32))]


@pytest.mark.parametrize("case", range(5))
def test_sort_rows_matches_stable_lexsort(tb, case):
    from trellis_cpp_b200 import ops
    name, coords = _cases()[case]
    got = ops.sort_rows(torch.from_numpy(np.ascontiguousarray(coords)).cuda()).cpu().numpy()
    ops.check_device()
    assert np.array_equal(got, _expected(coords)), name


def test_sort_rows_keeps_order_beyond_63_key_bits(tb):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(6)
    coords = rng.integers(-2 ** 31, 2 ** 31 - 1, size=(1000, 3), dtype=np.int64).astype(np.int32)
    got = ops.sort_rows(torch.from_numpy(coords).cuda()).cpu().numpy()
    assert np.array_equal(got, np.arange(1000, dtype=np.int32))


def test_sort_rows_empty(tb):
    from trellis_cpp_b200 import ops
    got = ops.sort_rows(torch.zeros((0, 3), dtype=torch.int32, device="cuda"))
    assert got.numel() == 0
