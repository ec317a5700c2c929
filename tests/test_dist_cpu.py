"""Multi-rank z-slab sharding on CPU: gloo ranks as processes (world 2 and 3).

Checks, without a GPU: the slabs partition the voxels, the halo exchange delivers exactly the
neighbouring planes' rows, and a conv computed independently on each rank's local rows
(owned + halo) equals the single-rank conv on every owned row (CPU oracle, bit for bit)."""
import os
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _worker(rank, world, init_file, result_dir):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import load_package
    load_package()
    import oracle
    from trellis_cpp_b200 import dist as tbdist, synth
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        coords = synth.coords_for("c1")
        n = coords.shape[0]
        rng = np.random.default_rng(3)
        feats = rng.standard_normal((n, 16)).astype(np.float32)
        w = (rng.standard_normal((8, 27, 16)) / 20).astype(np.float32)
        plan = tbdist.plan_slabs(coords, world, rank)
        gather = lambda t, idx: t.index_select(0, idx.long()).contiguous()   # noqa: E731
        scatter = lambda t, idx, src: t.index_copy_(0, idx.long(), src)       # noqa: E731
        own = torch.from_numpy(plan.own_local)
        assert np.array_equal(plan.local_rows()[plan.own_local], plan.owned)
        zl = coords[plan.local_rows(), -1]
        assert np.all(np.diff(zl) >= 0)                          # local rows ordered by z ...
        same_z = np.diff(zl) == 0
        assert np.all(np.diff(plan.local_rows())[same_z] > 0)   # ... and by input order within a plane
        assert np.array_equal(plan.own_local, np.arange(plan.own_local[0], plan.own_local[0] + plan.n_owned))
        x = torch.full((plan.n_local, 16), float("nan"), dtype=torch.float32)
        x[own] = torch.from_numpy(feats[plan.owned])
        tbdist.exchange_halo(plan, x, gather, scatter)
        halo = np.concatenate([plan.recv_lo, plan.recv_hi])
        halo_rows = plan.local_rows()[halo]
        ok_halo = np.array_equal(np.sort(halo_rows), np.sort(np.concatenate([plan.halo_lo, plan.halo_hi])))
        ok_halo = ok_halo and np.array_equal(x.numpy(), feats[plan.local_rows()])   # every local row filled
        # the started-then-finished form the GPU step uses to overlap the map build
        x2 = torch.full_like(x, float("nan"))
        x2[own] = 2 * x[own]
        handle = tbdist.exchange_halo(plan, x2, gather, scatter, wait=False)
        local = coords[plan.local_rows()]
        nbr_local = oracle.build_neighbor_table(local)          # work done while the transfer runs
        tbdist.finish_halo(handle)
        ok_halo = ok_halo and np.array_equal(x2.numpy(), 2 * feats[plan.local_rows()])
        out_local = oracle.submconv(nbr_local, x.numpy(), w)[plan.own_local]
        out_global = oracle.submconv(oracle.build_neighbor_table(coords), feats, w)[plan.owned]
        np.savez(os.path.join(result_dir, f"r{rank}.npz"), owned=plan.owned, ok_halo=ok_halo,
                 ok_conv=np.array_equal(out_local, out_global), n_halo=halo_rows.size)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_slab_halo_exchange_and_conv(world):
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "pg")
        mp.start_processes(_worker, args=(world, init_file, d), nprocs=world, start_method="spawn")
        owned = []
        for r in range(world):
            res = np.load(os.path.join(d, f"r{r}.npz"))
            assert bool(res["ok_halo"]), f"rank {r}: halo rows differ"
            assert bool(res["ok_conv"]), f"rank {r}: local conv differs from the single-rank conv"
            if 0 < r < world - 1 or world == 2:
                assert int(res["n_halo"]) > 0
            owned.append(res["owned"])
        allo = np.sort(np.concatenate(owned))
        assert np.array_equal(allo, np.arange(allo.size)), "slabs must partition the voxels"


def _worker_deep_halo(rank, world, init_file, result_dir):
    """Two stacked convs with a two-plane halo and no exchange between them: the first conv also
    computes the nearest halo plane on each side, which is all the second conv reads beyond the
    slab (the step SlabRunner runs through tb_dist_exchange / tb_dist_submconv_grow)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import load_package
    load_package()
    import oracle
    from trellis_cpp_b200 import dist as tbdist, synth
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world)
    try:
        coords = synth.coords_for("c1")
        n = coords.shape[0]
        rng = np.random.default_rng(5)
        feats = rng.standard_normal((n, 8)).astype(np.float32)
        w1 = (rng.standard_normal((8, 27, 8)) / 15).astype(np.float32)
        w2 = (rng.standard_normal((8, 27, 8)) / 15).astype(np.float32)
        plan = tbdist.plan_slabs(coords, world, rank, halo=2)
        gather = lambda t, idx: t.index_select(0, idx.long()).contiguous()   # noqa: E731
        scatter = lambda t, idx, src: t.index_copy_(0, idx.long(), src)       # noqa: E731
        x = torch.full((plan.n_local, 8), float("nan"), dtype=torch.float32)
        x[torch.from_numpy(plan.own_local)] = torch.from_numpy(feats[plan.owned])
        tbdist.exchange_halo(plan, x, gather, scatter)
        zl = coords[plan.local_rows(), -1]
        ok_halo = np.array_equal(x.numpy(), feats[plan.local_rows()])
        ok_halo = ok_halo and (rank == 0 or set(zl[plan.recv_lo]) == {plan.z_lo - 2, plan.z_lo - 1})
        nbr_local = oracle.build_neighbor_table(coords[plan.local_rows()])
        # conv 1 on the owned rows and the nearest halo plane; every other row of h stays NaN
        grow1 = (zl >= plan.z_lo - (1 if rank > 0 else 0)) & (zl < plan.z_hi + (1 if rank < world - 1 else 0))
        h_all = oracle.submconv(nbr_local, x.numpy(), w1, silu=True).astype(np.float32)
        h = np.full_like(h_all, np.nan)
        h[grow1] = h_all[grow1]
        out_local = oracle.submconv(nbr_local, h, w2)[plan.own_local]
        nbr_g = oracle.build_neighbor_table(coords)
        hg = oracle.submconv(nbr_g, feats, w1, silu=True).astype(np.float32)
        out_global = oracle.submconv(nbr_g, hg, w2)[plan.owned]
        np.savez(os.path.join(result_dir, f"r{rank}.npz"), owned=plan.owned, ok_halo=ok_halo,
                 ok_conv=np.array_equal(out_local, out_global))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_two_plane_halo_two_convs(world):
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "pg")
        mp.start_processes(_worker_deep_halo, args=(world, init_file, d), nprocs=world, start_method="spawn")
        owned = []
        for r in range(world):
            res = np.load(os.path.join(d, f"r{r}.npz"))
            assert bool(res["ok_halo"]), f"rank {r}: halo rows differ"
            assert bool(res["ok_conv"]), f"rank {r}: the two-conv stack differs from the single-rank stack"
            owned.append(res["owned"])
        assert np.array_equal(np.sort(np.concatenate(owned)), np.arange(sum(o.size for o in owned)))


def test_deep_halo_plan(tb):
    """halo=2: the rank holds two planes of each neighbour, sends its two edge planes, and a slab
    thinner than the halo is refused."""
    from trellis_cpp_b200 import dist as tbdist, synth
    coords = synth.coords_for("c2")
    z = coords[:, -1]
    world = 4
    plans = [tbdist.plan_slabs(coords, world, r, halo=2) for r in range(world)]
    for r, pl in enumerate(plans):
        zl = z[pl.local_rows()]
        if r > 0:
            assert set(zl[pl.recv_lo]) == {pl.z_lo - 2, pl.z_lo - 1}
            assert set(zl[pl.send_lo]) == {pl.z_lo, pl.z_lo + 1}
            # what rank r-1 sends up is what rank r receives from below, row for row
            prev = plans[r - 1]
            assert np.array_equal(prev.local_rows()[prev.send_hi], pl.local_rows()[pl.recv_lo])
        if r < world - 1:
            assert set(zl[pl.recv_hi]) == {pl.z_hi, pl.z_hi + 1}
    rng = np.random.default_rng(6)
    c = rng.integers(0, 6, (500, 3)).astype(np.int32)      # 6 planes over 4 ranks: slabs of 1-2 planes
    with pytest.raises(ValueError):
        tbdist.plan_slabs(c, 4, 0, halo=2)


def test_slab_bounds_balanced(tb):
    from trellis_cpp_b200 import dist as tbdist, synth
    coords = synth.coords_for("c2")
    for world in (2, 4, 8):
        sizes = [tbdist.plan_slabs(coords, world, r).n_owned for r in range(world)]
        assert sum(sizes) == coords.shape[0]
        assert max(sizes) < 1.15 * coords.shape[0] / world


def test_slab_plan_edge_cases(tb):
    from trellis_cpp_b200 import dist as tbdist
    rng = np.random.default_rng(4)
    c = rng.integers(0, 12, (2000, 3)).astype(np.int32)
    # one rank owns everything and has no halo
    p = tbdist.plan_slabs(c, 1, 0)
    assert p.n_owned == len(c) and p.n_local == len(c)
    assert p.send_lo.size == p.send_hi.size == p.recv_lo.size == p.recv_hi.size == 0
    # as many ranks as planes: one plane per slab, and every halo plane is a neighbour's owned plane
    world = 12
    plans = [tbdist.plan_slabs(c, world, r) for r in range(world)]
    assert all(pl.z_hi - pl.z_lo == 1 for pl in plans)
    assert np.array_equal(np.sort(np.concatenate([pl.owned for pl in plans])), np.arange(len(c)))
    for r in range(1, world):
        assert np.array_equal(plans[r].halo_lo, plans[r - 1].owned)
        assert plans[r].recv_lo.size == plans[r - 1].send_hi.size
    # more ranks than planes cannot be cut into slabs
    with pytest.raises(ValueError):
        tbdist.plan_slabs(c, 13, 0)


def test_host_cut_matches_library_cut(tb):
    """tb_zslab_cuts (the cut tb_dist_partition_zslab makes from its device histogram) equals
    the host planner's slab_bounds on shells, boxes, sparse planes and more ranks."""
    from trellis_cpp_b200 import dist as tbdist, ops, synth
    rng = np.random.default_rng(8)
    cases = [synth.coords_for("c1"), synth.coords_for("c2")]
    sparse = rng.integers(0, 40, (500, 3)).astype(np.int32)
    sparse[:, 2] = rng.choice([3, 4, 9, 17, 18, 30, 31, 32, 39], 500)       # empty planes between
    cases.append(sparse)
    cases.append(np.array([[0, 0, 5], [0, 0, 6], [1, 1, 7]], np.int32))
    for c in cases:
        z = c[:, -1].astype(np.int64)
        zmin = int(z.min()) - 3                                                # leading empty planes
        counts = np.bincount(z - zmin, minlength=int(z.max()) - zmin + 5)     # and trailing ones
        nplanes = int(z.max() - z.min() + 1)
        for world in (1, 2, 3, 4, 8, 16):
            if world > nplanes:
                with pytest.raises(ops.TBError):
                    ops.zslab_cuts(counts, zmin, world)
                continue
            assert np.array_equal(ops.zslab_cuts(counts, zmin, world), tbdist.slab_bounds(z, world)), world
