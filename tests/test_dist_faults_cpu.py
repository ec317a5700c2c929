"""Failure handling of the multi-rank halo exchange, on CPU (gloo ranks as processes, world 2).

The step's only cross-rank dependency is the halo exchange (dist.exchange_halo): each rank sends
its boundary planes and waits for its neighbours'. The failures are made on the host, never on
a GPU:
* a late rank (it sleeps before its exchange): the exchange still delivers the exact rows;
* a silent rank (alive, but its message never comes): the waiting rank's exchange raises within
  the process group's timeout instead of waiting for good;
* a dead rank (the process is gone before the exchange): the waiting rank's exchange raises.
The GPU step uses the same exchange over NCCL, where the process group's timeout ends a wait
for a rank that left in the same way."""
import datetime
import json
import os
import sys
import tempfile
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

TIMEOUT_S = 4


def _worker(rank, world, init_file, result_dir, mode):
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from conftest import load_package
    load_package()
    from trellis_cpp_b200 import dist as tbdist, synth
    dist.init_process_group("gloo", init_method=f"file://{init_file}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=TIMEOUT_S))
    res = {"rank": rank, "ok": False, "error": "", "elapsed": 0.0}
    try:
        coords = synth.coords_for("c1")
        feats = np.random.default_rng(5).standard_normal((coords.shape[0], 8)).astype(np.float32)
        plan = tbdist.plan_slabs(coords, world, rank)
        gather = lambda t, idx: t.index_select(0, idx.long()).contiguous()   # noqa: E731
        scatter = lambda t, idx, src: t.index_copy_(0, idx.long(), src)       # noqa: E731
        x = torch.full((plan.n_local, 8), float("nan"), dtype=torch.float32)
        x[torch.from_numpy(plan.own_local)] = torch.from_numpy(feats[plan.owned])
        faulty = rank == 1
        if faulty and mode == "late":
            time.sleep(1.5)
        if faulty and mode == "dead":
            os._exit(0)                             # gone without a word, as a crashed rank
        if faulty and mode == "silent":
            time.sleep(2 * TIMEOUT_S + 2)           # alive, but never sends
            res["ok"] = True
            return
        t0 = time.perf_counter()
        try:
            tbdist.exchange_halo(plan, x, gather, scatter)
            res["ok"] = bool(np.array_equal(x.numpy(), feats[plan.local_rows()]))
        except RuntimeError as e:                   # gloo reports the lost peer or the timeout
            res["error"] = str(e)[:300]
        res["elapsed"] = time.perf_counter() - t0
    finally:
        with open(os.path.join(result_dir, f"r{rank}.json"), "w") as f:
            json.dump(res, f)
        if mode == "late" or rank == 1:
            dist.destroy_process_group()


def _run(mode):
    with tempfile.TemporaryDirectory() as d:
        init_file = os.path.join(d, "pg")
        t0 = time.perf_counter()
        mp.start_processes(_worker, args=(2, init_file, d, mode), nprocs=2, start_method="spawn")
        wall = time.perf_counter() - t0
        out = {}
        for r in range(2):
            p = os.path.join(d, f"r{r}.json")
            out[r] = json.load(open(p)) if os.path.exists(p) else None
        return out, wall


def test_late_rank_still_exchanges_exactly():
    out, _ = _run("late")
    assert out[0]["ok"] and out[1]["ok"], out
    assert out[0]["elapsed"] > 1.0          # rank 0 waited for the late rank's rows


@pytest.mark.parametrize("mode", ["silent", "dead"])
def test_missing_rank_fails_the_exchange_within_the_timeout(mode):
    out, wall = _run(mode)
    r0 = out[0]
    assert r0 is not None and not r0["ok"], out
    assert r0["error"], "the waiting rank must see an error, not a silent result"
    assert r0["elapsed"] < TIMEOUT_S + 10, r0
