"""The z-slab step (dist.SlabRunner over the tb_dist_* C ABI) on two GPUs of one box, over NCCL:
every rank's owned rows after map + conv(SiLU) + conv must match the same rows of the one-GPU
step on the whole shell within the bf16 tolerance (the slab-local rows sum their 27 taps in
another order), the recorded CUDA-graph replay must equal the eager step bit for bit, and halo
rows poisoned with NaN before the step must be overwritten by the exchange. It runs only where
two GPUs are visible and TB_MULTI_GPU_TESTS=1 is set, so that a single-GPU test run never starts
NCCL ranks. The ranks are child processes with a short process-group timeout; each releases its
graph and communicator before destroying the group."""
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
        g = torch.Generator(device=dev).manual_seed(7)
        w1 = (torch.randn((64, 27, 64), device=dev, generator=g) / np.sqrt(27 * 64)).bfloat16()
        w2 = (torch.randn((64, 27, 64), device=dev, generator=g) / np.sqrt(27 * 64)).bfloat16()
        uid = [ops.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        runner = tbdist.SlabRunner(coords_np, 64, dev, g, uid[0])
        sl = runner.slab
        ob = int(sl.owned_begin)
        runner.feats[:ob] = float("nan")                     # halo rows: must come from the peer
        runner.feats[ob + runner.n_owned:] = float("nan")
        runner.step(w1, w2)
        torch.cuda.synchronize(dev)
        chk = runner.check_against_single_gpu(w1, w2)
        res.update(chk)
        res["max_rel"] = chk["max_abs"] / max(chk["max_ref"], 1e-30)
        res["n_halo"] = int(sl.n_halo_lo + sl.n_halo_hi)
        res["finite"] = bool(torch.isfinite(runner.out[runner.owned].float()).all())
        eager = runner.out[runner.owned].clone()
        runner.out.zero_()
        runner.capture(w1, w2)
        runner.replay()
        torch.cuda.synchronize(dev)
        res["replay_equal"] = bool(torch.equal(runner.out[runner.owned], eager))
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
        assert r["finite"], f"rank {r['rank']}: owned rows not finite (halo not received?)"
        assert r["max_rel"] < 1e-2, f"rank {r['rank']}: slab step differs from the one-GPU step: {r}"
        assert r["rows_bit_exact"] > 0.5 * r["rows_checked"], r      # most rows identical, the rest an ulp apart
        assert r["replay_equal"], f"rank {r['rank']}: graph replay differs from the eager step"
    assert sum(r["rows_checked"] for r in out) == 249154
