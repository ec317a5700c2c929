"""The allocation-free neighbor-map entry point, tb_build_neighbor_map_noalloc.

It exists for callers that cannot allocate device memory when they need a map (a framework
that serves every device buffer from its own pool, or code that must not call cudaMalloc
because it can synchronise the device). It builds the same map as tb_build_neighbor_map,
using a hash table compiled into the library as a static device array. These tests call it
through the C ABI twice in a row, on different inputs, and require each result to equal the
ordinary entry point's map bit for bit (maps are integer data; the tolerance is zero).

This file is collected last on purpose, and passes both on its own in a fresh process and
after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import random_voxels

pytestmark = pytest.mark.gpu

TB_ERR_INVALID_ARG = 1
TB_ERR_TOO_LARGE = 6


def _noalloc_map(lib, coords_t):
    n = coords_t.shape[0]
    out = torch.full((27 * n,), -7, dtype=torch.int32, device=coords_t.device)
    stream = torch.cuda.current_stream(coords_t.device).cuda_stream
    st = lib.tb_build_neighbor_map_noalloc(ctypes.c_void_p(stream), ctypes.c_void_p(coords_t.data_ptr()), n,
                                           coords_t.shape[1], ctypes.c_void_p(out.data_ptr()))
    assert st == 0, f"tb_build_neighbor_map_noalloc returned {st}"
    torch.cuda.synchronize()
    return out


def _inputs():
    from trellis_cpp_b200 import synth
    rng = np.random.default_rng(21)
    dups = rng.integers(0, 14, size=(9000, 3)).astype(np.int32)          # many duplicate rows
    # exactly the maximum size, so the table spans all of its slots and the cell after them;
    # a (-1,-1,-1) voxel has the all-ones key, which lives in that separate cell
    full = random_voxels(524288 - 1, 90, 22)
    full = np.concatenate([full[:1000], np.full((1, 3), -1, np.int32), full[1000:]])
    return [("c2 shell", synth.coords_for("c2")),                        # 249K voxels, [N,4]
            ("random with duplicates", dups),
            ("maximum size with an all-ones key", full),
            ("small box", random_voxels(3000, 30, 4))]


def test_noalloc_matches_allocating_entry_point_twice_in_a_row(tb):
    from trellis_cpp_b200 import _lib, ops
    lib = _lib.load()
    cases = _inputs()
    # two passes over the cases: every call runs right after a call on different coordinates,
    # so a table left over from the previous call would show up as a wrong map
    for _round in range(2):
        for name, coords in cases:
            c = torch.from_numpy(np.ascontiguousarray(coords)).cuda()
            got = _noalloc_map(lib, c)
            want = ops.build_neighbor_table(c)
            ops.check_device()
            assert torch.equal(got, want), f"{name}: map differs from tb_build_neighbor_map"


def test_noalloc_rejects_sizes_above_the_limit(tb):
    from trellis_cpp_b200 import _lib
    lib = _lib.load()
    n = 524288 + 1
    coords = torch.zeros((n, 3), dtype=torch.int32, device="cuda")
    out = torch.zeros(16, dtype=torch.int32, device="cuda")
    st = lib.tb_build_neighbor_map_noalloc(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                           ctypes.c_void_p(coords.data_ptr()), n, 3,
                                           ctypes.c_void_p(out.data_ptr()))
    assert st == TB_ERR_TOO_LARGE


def test_noalloc_rejects_host_memory(tb):
    """Coordinates in (pinned) host memory are refused before anything is launched."""
    from trellis_cpp_b200 import _lib
    lib = _lib.load()
    coords = torch.zeros((64, 3), dtype=torch.int32).pin_memory()
    out = torch.zeros(27 * 64, dtype=torch.int32, device="cuda")
    st = lib.tb_build_neighbor_map_noalloc(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                           ctypes.c_void_p(coords.data_ptr()), 64, 3,
                                           ctypes.c_void_p(out.data_ptr()))
    assert st == TB_ERR_INVALID_ARG
