"""The bounded-wait abort path of the tensor-core conv, run on purpose without hanging anything.

Every mbarrier wait in the conv kernels gives up after a clock limit (about 2 s), sets the
context's device error word and leaves the kernel through its abort path (TMA copies allowed to
land, MMAs drained, TMEM freed). A test-only hook of the pair kernel shortens that limit to about
1 ms and makes one epilogue warp of every CTA pair withhold one arrive after its first tile, so
the next waits on that barrier run out. The test checks that the launch returns, that
tb_ctx_check_device reports the timeout (and clears it), and that the next normal conv on the
same context is correct. No GPU fault, trap or endless loop is involved: the waits end by
themselves."""
import ctypes
import time

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_withheld_arrive_times_out_and_the_context_recovers(tb):
    from trellis_cpp_b200 import _lib, ops, synth
    lib = _lib.load()
    hook = lib.tb_debug_pair_withhold_arrive
    hook.argtypes = [ctypes.c_int, ctypes.c_longlong]
    hook.restype = None
    coords = torch.from_numpy(synth.coords_for("c2")).cuda()     # 249K voxels: >= 2 tiles per CTA pair
    n = coords.shape[0]
    nbr = ops.build_neighbor_table(coords)
    g = torch.Generator(device="cuda").manual_seed(31)
    f = torch.randn((n, 64), device="cuda", generator=g).bfloat16()
    w = (torch.randn((64, 27, 64), device="cuda", generator=g) / 40).bfloat16()
    good = ops.sparse_submconv(f, nbr, w, None, out_dtype=torch.float32)
    ops.check_device()
    hook(1, 2_000_000)                                            # ~1 ms wait limit, one arrive withheld
    try:
        t0 = time.perf_counter()
        ops.sparse_submconv(f, nbr, w, None, out_dtype=torch.float32)
        with pytest.raises(ops.TBError) as e:
            ops.check_device()
        dt = time.perf_counter() - t0
    finally:
        hook(0, 0)
    assert e.value.status == 5 and "timed out" in str(e.value)
    assert dt < 30.0
    ops.check_device()                                            # the error word was cleared
    again = ops.sparse_submconv(f, nbr, w, None, out_dtype=torch.float32)
    ops.check_device()
    assert torch.equal(again, good)
