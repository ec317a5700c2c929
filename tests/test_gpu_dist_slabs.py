"""The multi-GPU z-slab calls (tb_dist_*) on one GPU, through the C ABI.

A dist made without a communicator exchanges nothing and takes the halo rows from the caller, so
one process can play every rank of a `world`-rank split in turn. For each rank: the partition
(cut, local rows in z order, contiguous owned and edge ranges), the slab's neighbor map (the
global map of every owned row, with the taps relabelled to the (z, x, y) local axes) and a conv
on the owned rows, which must equal the single-GPU conv of the same rows up to fp32
accumulation order (1e-5 relative with fp32 outputs, 1e-2 with bf16 ones)."""
import numpy as np
import pytest
import torch

from conftest import max_rel

pytestmark = pytest.mark.gpu


def _global_tap(tl):
    return ((tl // 3) % 3) * 9 + (tl % 3) * 3 + tl // 9


@pytest.mark.parametrize("name,world", [("c2", 1), ("c2", 2), ("c2", 5), ("c1", 8), ("c1", 16), ("c1", 30), ("c5_32", 3)])
def test_slab_partition_map_and_conv(tb, name, world):
    from trellis_cpp_b200 import dist as tbdist, ops, synth
    coords_np = synth.coords_for(name)
    n = coords_np.shape[0]
    dev = torch.device("cuda", 0)
    coords = torch.from_numpy(coords_np).to(dev)
    nbr = ops.build_neighbor_table(coords)
    nbr_h = nbr.view(27, n).cpu().numpy()
    g = torch.Generator(device=dev).manual_seed(12)
    f = torch.randn((n, 64), device=dev, generator=g).bfloat16()
    w = (torch.randn((64, 27, 64), device=dev, generator=g) / np.sqrt(27 * 64)).bfloat16()
    b = 0.1 * torch.randn(64, device=dev, generator=g)
    ref = ops.sparse_submconv(f, nbr, w, b, epi="silu", out_dtype=torch.float32)
    ref16 = ops.sparse_submconv(f, nbr, w, b, epi="silu")
    z = coords_np[:, -1]
    owned_all = []
    for rank in range(world):
        d = ops.Dist(dev, rank, world)          # no communicator: the halo rows come from here
        try:
            sl = d.partition(coords)
            plan = tbdist.plan_slabs(coords_np, world, rank)
            rows = d.local_rows().cpu().numpy()
            # the cut and the local order are the host planner's
            assert (sl.z_lo, sl.z_hi) == (plan.z_lo, plan.z_hi)
            assert np.array_equal(rows, plan.local_rows())
            ob, no = sl.owned_begin, sl.n_owned
            assert np.array_equal(rows[ob:ob + no], plan.owned)
            assert sl.n_halo_lo == plan.recv_lo.size and sl.n_halo_hi == plan.recv_hi.size
            assert np.all(z[rows[ob:ob + sl.n_edge_lo]] == sl.z_lo)
            assert np.all(z[rows[ob + no - sl.n_edge_hi:ob + no]] == sl.z_hi - 1)
            owned_all.append(rows[ob:ob + no])
            # the slab's map: for every owned row, local tap t' is the global tap _global_tap(t')
            d.build_map()
            lm = d.local_map().view(27, sl.n_local).cpu().numpy()
            own = np.arange(ob, ob + no)
            for tl in range(27):
                loc = lm[tl, own]
                got = np.where(loc == sl.n_local, n, rows[np.minimum(loc, sl.n_local - 1)])
                assert np.array_equal(got, nbr_h[_global_tap(tl), rows[own]]), (rank, tl)
            pairs = d.count_valid_pairs()
            assert pairs == int((nbr_h[:, rows[own]] != n).sum())
            # a conv on the owned rows; the halo rows are given (nothing is exchanged)
            rows_t = torch.from_numpy(rows).to(dev).long()
            fl = f[rows_t].contiguous()
            out = torch.full((sl.n_local, 64), float("nan"), device=dev)
            d.submconv(fl, w, b, epi="silu", out_dtype=torch.float32, out=out)
            out16 = d.submconv(fl, w, b, epi="silu")
            ops.check_device()
            o = out[ob:ob + no].cpu().numpy()
            assert not np.isnan(o).any()
            assert max_rel(o, ref[rows_t[ob:ob + no]].cpu().numpy()) < 1e-5
            assert max_rel(out16[ob:ob + no].float().cpu().numpy(),
                           ref16[rows_t[ob:ob + no]].float().cpu().numpy()) < 1e-2
            # halo rows of the output are left alone
            if sl.n_halo_lo:
                assert torch.isnan(out[:ob]).all()
        finally:
            d.close()
    allo = np.sort(np.concatenate(owned_all))
    assert np.array_equal(allo, np.arange(n)), "the slabs must partition the voxels"


@pytest.mark.parametrize("name,world", [("c2", 2), ("c2", 5), ("c1", 8), ("c5_32", 3)])
def test_two_plane_halo_stack(tb, name, world):
    """halo_planes = 2 and no exchange between two convs (tb_dist_submconv_grow): conv 1 over the
    owned rows and the nearest halo plane per side, conv 2 over the owned rows, against the
    single-GPU stack; the partition is the host planner's with halo=2, and rows outside each
    conv's range are left untouched."""
    from trellis_cpp_b200 import dist as tbdist, ops, synth
    coords_np = synth.coords_for(name)
    n = coords_np.shape[0]
    dev = torch.device("cuda", 0)
    coords = torch.from_numpy(coords_np).to(dev)
    nbr = ops.build_neighbor_table(coords)
    g = torch.Generator(device=dev).manual_seed(13)
    f = torch.randn((n, 64), device=dev, generator=g).bfloat16()
    w1 = (torch.randn((64, 27, 64), device=dev, generator=g) / np.sqrt(27 * 64)).bfloat16()
    w2 = (torch.randn((64, 27, 64), device=dev, generator=g) / np.sqrt(27 * 64)).bfloat16()
    h_ref = ops.sparse_submconv(f, nbr, w1, None, epi="silu")
    ref = ops.sparse_submconv(h_ref, nbr, w2, None, out_dtype=torch.float32)
    z = coords_np[:, -1]
    for rank in range(world):
        d = ops.Dist(dev, rank, world, halo_planes=2)
        try:
            sl = d.partition(coords)
            plan = tbdist.plan_slabs(coords_np, world, rank, halo=2)
            rows = d.local_rows().cpu().numpy()
            assert np.array_equal(rows, plan.local_rows())
            assert sl.n_halo_lo == plan.recv_lo.size and sl.n_halo_hi == plan.recv_hi.size
            assert sl.n_edge_lo == plan.send_lo.size or rank == 0
            d.build_map()
            rows_t = torch.from_numpy(rows).to(dev).long()
            fl = f[rows_t].contiguous()                       # halo rows given (nothing exchanged)
            w1l, w2l = d.local_weight(w1), d.local_weight(w2)
            h = torch.full((sl.n_local, 64), float("nan"), device=dev).bfloat16()
            d.submconv_grow(1, fl, w1l, None, epi="silu", out=h)
            out = torch.full((sl.n_local, 64), float("nan"), device=dev)
            d.submconv_grow(0, h, w2l, None, out_dtype=torch.float32, out=out)
            ops.check_device()
            zl = z[rows]
            grown = (zl >= sl.z_lo - (1 if rank > 0 else 0)) & (zl < sl.z_hi + (1 if rank < world - 1 else 0))
            hc = h.float().cpu().numpy()
            assert not np.isnan(hc[grown]).any() and np.isnan(hc[~grown]).all()
            assert max_rel(hc[grown], h_ref[rows_t[torch.from_numpy(grown).to(dev)]].float().cpu().numpy()) < 1e-2
            ob, no = sl.owned_begin, sl.n_owned
            o = out.cpu().numpy()
            assert np.isnan(o[:ob]).all() and np.isnan(o[ob + no:]).all()
            assert max_rel(o[ob:ob + no], ref[rows_t[ob:ob + no]].cpu().numpy()) < 2e-2
            with pytest.raises(ops.TBError):
                d.submconv_grow(2, fl, w1l, None, out=h)      # grow must stay below the halo depth
        finally:
            d.close()


def test_dist_rejects_thin_slabs_for_deep_halo(tb):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(9)
    c = torch.from_numpy(rng.integers(0, 6, (500, 3)).astype(np.int32)).cuda()
    d = ops.Dist(torch.device("cuda", 0), 0, 4, halo_planes=2)
    try:
        with pytest.raises(ops.TBError):
            d.partition(c)
    finally:
        d.close()


def test_dist_rejects_too_many_ranks(tb):
    from trellis_cpp_b200 import ops
    c = torch.tensor([[0, 0, 0], [1, 0, 1], [0, 1, 2]], dtype=torch.int32, device="cuda")
    d = ops.Dist(torch.device("cuda", 0), 0, 4)
    try:
        with pytest.raises(ops.TBError):
            d.partition(c)
        with pytest.raises(ops.TBError):
            d.build_map()                     # no partition yet
    finally:
        d.close()
