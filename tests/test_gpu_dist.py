"""The z-slab step (dist.SlabRunner) on two GPUs of one box, over NCCL: every rank's owned rows
after map + conv(SiLU) + conv must equal the same rows of the one-GPU step on the whole shell,
bit for bit (the pair kernel sums each row's taps in a fixed order, wherever the row sits), for
the eager step and for the recorded CUDA-graph replay. It runs only where two GPUs are visible
and TB_MULTI_GPU_TESTS=1 is set, so that a single-GPU test run never starts NCCL ranks. The
ranks are child processes with a short process-group timeout; each releases its graph before
destroying the group."""
import datetime
import json
import os
import sys
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT

pytestmark = pytest.mark.gpu

WORKLOAD = "c2"          # 250 K-voxel res-256 shell: planes on both sides of every slab cut


def _rank(rank, world, init_file, result_dir):
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import load_package
    load_package()
    from trellis_cpp_b200 import dist as tbdist, ops, synth
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    res = {"rank": rank}
    runner = None
    try:
        coords_np = synth.coords_for(WORKLOAD)
        n = coords_np.shape[0]
        g = torch.Generator(device=dev).manual_seed(7)
        feats = torch.randn((n, 64), device=dev, generator=g).bfloat16()
        w1 = (torch.randn((64, 27, 64), device=dev, generator=g) / np.sqrt(27 * 64)).bfloat16()
        w2 = (torch.randn((64, 27, 64), device=dev, generator=g) / np.sqrt(27 * 64)).bfloat16()
        # the one-GPU step on the whole shell
        c_all = torch.from_numpy(coords_np).to(dev)
        nbr = ops.build_neighbor_table(c_all)
        h = ops.sparse_submconv(feats, nbr, w1, None, epi="silu")
        ref = ops.sparse_submconv(h, nbr, w2, None)
        # the slab step: owned rows from the same features, halo rows filled by the exchange
        runner = tbdist.SlabRunner(coords_np, 64, dev, g)
        local = torch.from_numpy(runner.plan.local_rows()).to(dev)
        runner.feats.copy_(feats[local])
        runner.feats[torch.from_numpy(np.concatenate([runner.plan.recv_lo, runner.plan.recv_hi])).to(dev)
                     .long()] = float("nan")
        runner.step(w1, w2)
        torch.cuda.synchronize(dev)
        own = torch.from_numpy(runner.plan.own_local).to(dev)
        owned = torch.from_numpy(runner.plan.owned).to(dev)
        res["eager_equal"] = bool(torch.equal(runner.out[own], ref[owned]))
        res["n_owned"] = int(own.numel())
        res["n_halo"] = int(runner.plan.recv_lo.size + runner.plan.recv_hi.size)
        runner.out.zero_()
        runner.capture(w1, w2)
        runner.replay()
        torch.cuda.synchronize(dev)
        res["replay_equal"] = bool(torch.equal(runner.out[own], ref[owned]))
        ops.check_device()
    finally:
        if runner is not None:
            runner.close()
        with open(os.path.join(result_dir, f"r{rank}.json"), "w") as f:
            json.dump(res, f)
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2 or os.environ.get("TB_MULTI_GPU_TESTS") != "1",
                    reason="needs two GPUs and TB_MULTI_GPU_TESTS=1")
def test_two_rank_slab_step_matches_one_gpu(tb):
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_rank, args=(2, os.path.join(d, "pg"), d), nprocs=2, start_method="spawn")
        out = [json.load(open(os.path.join(d, f"r{r}.json"))) for r in range(2)]
    for r in out:
        assert r["n_halo"] > 0, r
        assert r["eager_equal"], f"rank {r['rank']}: eager slab step differs from the one-GPU step"
        assert r["replay_equal"], f"rank {r['rank']}: graph replay differs from the one-GPU step"
