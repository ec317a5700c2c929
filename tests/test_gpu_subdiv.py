"""GPU subdivide / channel-to-spatial gather / bias+act vs the reference semantics."""
import numpy as np
import pytest
import torch

import oracle
from conftest import max_rel

pytestmark = pytest.mark.gpu


def _sub(coords, mask, max_children=None):
    from trellis_cpp_b200 import ops
    c = torch.from_numpy(np.ascontiguousarray(coords, dtype=np.int32)).cuda()
    m = torch.from_numpy(np.ascontiguousarray(mask, dtype=np.uint8)).cuda()
    child, gidx, mstart = ops.subdivide(c, m, max_children)
    return child.cpu().numpy(), gidx.cpu().numpy(), mstart.cpu().numpy()


def test_golden_c2s_subdivide(tb, golden):
    g = golden["c2s"]
    child, gidx, mstart = _sub(g["coords"], g["mask"])
    assert np.array_equal(child, g["new_coords"])
    assert np.array_equal(gidx, g["gather_octant"] + 8 * g["gather_parent"])
    assert mstart[-1] == child.shape[0]


@pytest.mark.parametrize("p", [0.0, 0.3, 1.0])
def test_random_masks_vs_oracle(tb, p):
    rng = np.random.default_rng(int(p * 10))
    c = rng.integers(0, 500, size=(10007, 4)).astype(np.int32)
    c[:, 0] = rng.integers(0, 3, 10007)
    mask = (rng.random((10007, 8)) < p).astype(np.uint8) * rng.integers(1, 255, (10007, 8)).astype(np.uint8)
    child, gidx, mstart = _sub(c, mask)
    oc, og, om = oracle.subdivide(c, mask != 0)
    assert np.array_equal(child, oc) and np.array_equal(gidx, og) and np.array_equal(mstart, om)


def test_c3_full_size(tb):
    from trellis_cpp_b200 import synth
    c = synth.coords_for("c3")
    mask = synth.c3_mask(c)
    child, gidx, mstart = _sub(c, mask)
    oc, og, om = oracle.subdivide(c, mask)
    assert np.array_equal(child, oc) and np.array_equal(gidx, og) and np.array_equal(mstart, om)


def test_max_children_exceeded(tb):
    from trellis_cpp_b200 import ops
    c = np.zeros((10, 3), np.int32)
    c[:, 0] = np.arange(10)
    with pytest.raises(ops.TBError) as e:
        _sub(c, np.ones((10, 8), np.uint8), max_children=20)
    assert e.value.status == 6


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16, torch.float16])
def test_c2s_gather(tb, dt):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(3)
    n, c = 700, 24
    src = torch.from_numpy(rng.standard_normal((n, 8 * c)).astype(np.float32)).cuda().to(dt)
    gidx = torch.from_numpy(np.sort(rng.choice(8 * n, 2000, replace=False)).astype(np.int32)).cuda()
    out = ops.c2s_gather(src, gidx, c)
    ref = oracle.c2s_gather(src.float().cpu().numpy(), gidx.cpu().numpy(), c)
    assert np.array_equal(out.float().cpu().numpy(), ref)


@pytest.mark.parametrize("dt", [torch.float32, torch.bfloat16])
def test_bias_act(tb, dt):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(4)
    x = torch.from_numpy(rng.standard_normal((999, 48)).astype(np.float32)).cuda().to(dt)
    b = torch.from_numpy(rng.standard_normal(48).astype(np.float32)).cuda()
    ref = oracle.silu(x.float().cpu().numpy().astype(np.float64) + b.cpu().numpy())
    ops.bias_act(x, b, "silu")
    assert max_rel(x.float().cpu().numpy(), ref) < (1e-6 if dt == torch.float32 else 1e-2)


@pytest.mark.parametrize("c,dt", [(64, torch.bfloat16), (16, torch.float32), (3, torch.float32)])
def test_gather_and_scatter_rows(tb, c, dt):
    # the halo packing of the multi-GPU step: gather rows into a contiguous buffer, scatter a
    # received buffer back to its row positions (row sizes with and without 16-byte vectors)
    from trellis_cpp_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(c)
    src = torch.randn((5000, c), device="cuda", generator=g).to(dt)
    rows = torch.randperm(5000, device="cuda", generator=g)[:1234].to(torch.int32)
    packed = ops.gather_rows(src, rows)
    assert torch.equal(packed, src[rows.long()])
    dst = torch.zeros_like(src)
    ops.scatter_rows(dst, rows, packed)
    ops.check_device()
    expect = torch.zeros_like(src)
    expect[rows.long()] = src[rows.long()]
    assert torch.equal(dst, expect)
