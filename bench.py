#!/usr/bin/env python3
"""Benchmark of the sparse submanifold-conv path on B200 (one JSON line on rank 0).

Workload: the res-1024 noisy-sphere shell, ~4.9M active voxels, two
stacked 3x3x3 submanifold convs at Cin=Cout=64, bf16 operands, fp32 accumulation.
One step = build the neighbor map from the coordinates + conv(SiLU) + conv, with coords,
features and weights resident in HBM. Metric: active voxels/s (whole job).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 (torchrun, one rank per GPU): the voxels are cut into z-slabs at voxel-count
quantiles; each rank owns one slab and holds two planes of each neighbour, exchanged over NCCL
(send/recv) once per step while it builds its local neighbor map; conv 1 computes its owned rows
and the nearest halo plane on each side, conv 2 its owned rows. Total work is fixed as N grows
("scaling": "strong").

`--impl reference` times the reference algorithm's CPU implementation (the oracle port in
oracle/, all host threads) on a bounded sample of the same workload.

`--op c2s` measures one SparseResBlockC2S3d up-block (src/sparse.cpp:172-336) on the config-3
parents (res-256 noisy shell) with its seeded child mask, Cin=256 -> Cout=128 bf16; metric
children/s, roofline of conv1 (256 -> 8*128 channels, the block's dominant kernel).

`--op decode` measures the sparse decoder UNet (decode_unet, src/shape_decoder.cpp:79-117) with
the reference's stage table (widths 1024/512/256/128, 4/16/8/4 ConvNeXt blocks, C2S blocks, output
64 -> 7) and random weights, on a res-32 noisy shell grown to res 512 by seeded shell-following
masks (the texture decoder's guided path); metric output voxels/s.

`--op mesh` measures dual_grid_to_mesh (src/dual_grid.cpp:16-56) on the config-4 shell taken as
the decoded voxels (res 1024) with seeded decoder-head fields; metric voxels/s; CPU baseline = the
reference's own dual_grid_to_mesh compiled from its sources (oracle/_ref) where it was built.

`--op convnext` measures one sparse ConvNeXt block instead (src/sparse.cpp:94-137 on the same
shell): the conv into an fp32 h, then the fused LayerNorm + Linear C->4C + SiLU + Linear 4C->C +
residual tail; metric voxels/s of the block, roofline of the tail kernel (HBM-bound).
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import subprocess
import sys
import threading
import time
import zlib

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.join(ROOT, "trellis.cpp_b200")
WORKLOAD = "c4"
CI = CO = 64
METRIC = "active voxels/s, 3^3 submanifold conv x2 + neighbor map, ~4.9M voxels C=64 (config 4)"


def _load_package():
    if "trellis_cpp_b200" in sys.modules:
        return sys.modules["trellis_cpp_b200"]
    spec = importlib.util.spec_from_file_location(
        "trellis_cpp_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["trellis_cpp_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


def _peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("bf16_tflops", 1590.0), d.get("hbm_gbs", 6650.0), "measured"
    return 1590.0, 6650.0, "fallback"


def _cpu_model() -> str:
    """The host CPU's model name (from /proc/cpuinfo), or "" where it cannot be read."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return ""


def _emit(line: dict) -> None:
    """Print the bench's JSON line; a CPU baseline also names the host CPU it ran on."""
    if isinstance(line.get("cpu_baseline"), dict):
        line["cpu_baseline"].setdefault("cpu", _cpu_model())
    print(json.dumps(line), flush=True)


def _profile_traffic(name="submconv_pair_c4.md"):
    """DRAM bytes per launch at full size from a committed ncu summary, or None."""
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.strip().startswith("dram_bytes_per_launch_full_size"):
            try:
                return int(line.split("=")[1].strip().strip("`"))
            except (IndexError, ValueError):
                return None
    return None


class ClockSampler:
    """nvidia-smi clock/throttle samples of one GPU (by UUID) while running."""

    FIELDS = ["uuid", "clocks.sm", "clocks.max.sm", "power.draw", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap"]

    def __init__(self, uuid: str):
        self.uuid = uuid
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + ",".join(self.FIELDS), "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == len(self.FIELDS) and self.uuid in parts[0]:
                self.rows.append(parts)

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in self.rows for k in range(4) if r[4 + k] == "Active"})
        loaded = [s for s in sm if s > 0.5 * (max(mx) if mx else 1)] or sm
        return {"sm_mhz": float(np.median(loaded)) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ----------------------------------------------------------------------------- CPU legs
def cpu_reference_step(coords, nbr_full, feats, wt1, wt2, sample, nthreads):
    """One bounded CPU step of the reference algorithm: the full neighbor map, single-threaded as
    src/sparse.cpp:21-39 is (the reference's own function compiled from its source where
    oracle/_ref holds it, else the oracle port), and both convs (oracle port, fp32, all threads)
    on `sample` output rows. Returns seconds per voxel."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    n = coords.shape[0]
    t0 = time.perf_counter()
    if oracle.ref_nbr_available():
        oracle.ref_build_neighbor_table(coords)      # the reference's own std::unordered_map loop
    else:
        oracle.build_neighbor_table(coords)
    t_map = time.perf_counter() - t0
    row0 = (n - sample) // 2
    h = feats.copy()          # rows outside the sample stand in for the first conv's output
    t0 = time.perf_counter()
    oracle.submconv_f32_mt_range(nbr_full, feats, wt1, row0, sample, silu=True, nthreads=nthreads, out=h)
    # the second conv reads neighbors of the sample rows; those rows' inputs are computed by
    # the first conv in a full run, here they reuse the first conv's sample output region
    oracle.submconv_f32_mt_range(nbr_full, h, wt2, row0, sample, nthreads=nthreads)
    t_conv = time.perf_counter() - t0
    return t_map / n + t_conv / sample, t_map, t_conv


def _map_kind():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    return ("the reference's own build_neighbor_table, compiled from src/sparse.cpp"
            if oracle.ref_nbr_available() else "the oracle port of build_neighbor_table")


def _cpu_inputs(coords):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    rng = np.random.default_rng(1)
    n = coords.shape[0]
    feats = rng.standard_normal((n, CI), dtype=np.float32)
    w1 = (rng.standard_normal((CO, 27, CI)) / np.sqrt(27 * CI)).astype(np.float32)
    w2 = (rng.standard_normal((CO, 27, CO)) / np.sqrt(27 * CO)).astype(np.float32)
    nbr = oracle.build_neighbor_table(coords)
    return feats, oracle.weight_tap_major(w1), oracle.weight_tap_major(w2), nbr


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    pkg = _load_package()
    from trellis_cpp_b200 import synth
    del pkg
    coords = synth.coords_for(WORKLOAD)
    n = coords.shape[0]
    nthreads = os.cpu_count() or 1
    feats, wt1, wt2, nbr = _cpu_inputs(coords)
    sample = min(n, 1 << 19)
    for _ in range(max(0, min(args.warmup, 1))):
        cpu_reference_step(coords, nbr, feats, wt1, wt2, min(sample, 1 << 16), nthreads)
    per_voxel = []
    for _ in range(max(1, min(args.steps, 3))):
        spv, _, _ = cpu_reference_step(coords, nbr, feats, wt1, wt2, sample, nthreads)
        per_voxel.append(spv)
    spv = float(np.median(per_voxel))
    value = 1.0 / spv
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "voxels/s", "n_gpus": args.gpus,
        "steps": len(per_voxel), "warmup": min(args.warmup, 1), "ms_per_step": spv * n * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded noisy shell, random N(0,1) features, N(0,1/(27*64)) weights)",
        "config": {"workload": "c4: res-1024 noisy shell, map + conv(SiLU) + conv, C=64", "voxels": n},
        "cpu_baseline": {"value": value, "unit": "voxels/s", "cores": nthreads, "kind": "port",
                         "sample": f"full single-threaded neighbor map over {n} voxels ({_map_kind()}) + both "
                                   f"fp32 convs (oracle port) on {sample} output rows (threads={nthreads}); "
                                   f"per-voxel times summed"},
        "e2e": {"value": value, "unit": "voxels/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    _emit(line)
    return 0


# ----------------------------------------------------------------------------- GPU arm
def run_gpu(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    _load_package()
    from trellis_cpp_b200 import ops, synth

    coords_np = synth.coords_for(args.workload)
    n_total = coords_np.shape[0]
    g = torch.Generator(device=dev).manual_seed(1234)
    w1 = (torch.randn((CO, 27, CI), device=dev, generator=g) / np.sqrt(27 * CI)).bfloat16()
    w2 = (torch.randn((CO, 27, CO), device=dev, generator=g) / np.sqrt(27 * CO)).bfloat16()

    if world > 1:
        from trellis_cpp_b200 import dist as tbdist
        uid = [ops.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        runner = tbdist.SlabRunner(coords_np, CI, dev, g, uid[0])
        step = lambda: runner.step(w1, w2)  # noqa: E731  (replaced by the recorded graph below)
        n_local = runner.n_owned
        nbr_for_flops = None
    else:
        coords = torch.from_numpy(coords_np).to(dev)
        feats = torch.randn((n_total, CI), device=dev, generator=g).bfloat16()
        nbr = torch.empty(27 * n_total, dtype=torch.int32, device=dev)
        h = torch.empty((n_total, CO), dtype=torch.bfloat16, device=dev)
        out = torch.empty((n_total, CO), dtype=torch.bfloat16, device=dev)
        conv_events = []

        def step(record=False):
            ops.build_neighbor_table(coords, out=nbr)
            if record:
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                e2 = torch.cuda.Event(enable_timing=True)
                e0.record()
                ops.sparse_submconv(feats, nbr, w1, None, epi="silu", out=h)
                e1.record()
                ops.sparse_submconv(h, nbr, w2, None, out=out)
                e2.record()
                conv_events.append((e0, e1, e2))
            else:
                ops.sparse_submconv(feats, nbr, w1, None, epi="silu", out=h)
                ops.sparse_submconv(h, nbr, w2, None, out=out)
        n_local = n_total
        nbr_for_flops = nbr

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        # each rank replays one CUDA graph per step (the NCCL halo exchange beside the map, both convs)
        runner.capture(w1, w2)
        step = runner.replay
    if nbr_for_flops is not None:
        pairs = ops.count_valid_pairs(nbr_for_flops, n_total)
    else:
        pairs = runner.count_valid_pairs()
    ops.check_device()

    uuid = str(torch.cuda.get_device_properties(dev).uuid)
    sampler = ClockSampler(uuid)
    sampler.start()
    time.sleep(0.8)   # nvidia-smi needs a moment before its first sample
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(args.steps):
        if world > 1:
            step()
        else:
            step(record=True)
    t_end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    sampler.stop()
    ms_total = t_start.elapsed_time(t_end)
    if world > 1:
        t = torch.tensor([ms_total], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
        allp = torch.tensor([pairs], device=dev, dtype=torch.int64)
        dist.all_reduce(allp)
        pairs_total = int(allp.item())
    else:
        pairs_total = pairs
    ops.check_device()
    ms_step = ms_total / args.steps
    value = n_total / (ms_step / 1e3)
    flops_step = 2 * 2.0 * CI * CO * pairs_total          # two convs, algorithmic (present pairs)
    eff_tflops = flops_step / (ms_step / 1e3) / 1e12
    peak_tf, peak_bw, peak_kind = _peaks()

    roofline = None
    kernel_stats = {}
    if world == 1:
        c1 = [a.elapsed_time(b) for a, b, _ in conv_events]
        c2 = [b.elapsed_time(c) for _, b, c in conv_events]
        conv_ms = float(np.mean(c1 + c2))
        flops_launch = 2.0 * CI * CO * pairs
        achieved = flops_launch / (conv_ms / 1e3) / 1e12
        traffic = _profile_traffic()
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                    "frac": achieved / peak_tf, "traffic": traffic,
                    "peak_source": f"{peak_kind} bf16_tflops (burst)", "kernel": "k_submconv_pair",
                    "flops_per_launch": flops_launch}
        kernel_stats = {"conv_ms_avg": conv_ms, "conv1_ms": float(np.mean(c1)), "conv2_ms": float(np.mean(c2)),
                        "map_ms_est": ms_step - float(np.mean(c1)) - float(np.mean(c2))}

    parity = None
    if world > 1:
        # per-rank times of the map (with the halo exchange beside it) and of each conv (eager steps
        # after the timed replays; conv 1 also computes the nearest halo plane on each side), slowest rank
        w1l, w2l = runner.local_weight(w1), runner.local_weight(w2)
        evs = []
        for _ in range(max(3, min(args.steps, 10))):
            e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            e[0].record()
            runner.dist.exchange(runner.feats)
            runner.dist.build_map()
            e[1].record()
            runner.dist.submconv_grow(1, runner.feats, w1l, None, epi="silu", out=runner.h)
            e[2].record()
            runner.dist.submconv_grow(0, runner.h, w2l, None, out=runner.out)
            e[3].record()
            evs.append(e)
        torch.cuda.synchronize()
        map_ms = float(np.mean([e[0].elapsed_time(e[1]) for e in evs]))
        conv_ms = float(np.mean([e[1].elapsed_time(e[2]) for e in evs] + [e[2].elapsed_time(e[3]) for e in evs]))
        tm = torch.tensor([conv_ms, map_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        conv_ms_max, map_ms_max = float(tm[0].item()), float(tm[1].item())
        flops_gpu = 2.0 * CI * CO * pairs_total / world        # one conv's algorithmic FLOPs per GPU
        achieved = flops_gpu / (conv_ms_max / 1e3) / 1e12
        roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                    "frac": achieved / peak_tf, "traffic": None, "peak_source": f"{peak_kind} bf16_tflops (burst)",
                    "kernel": "k_submconv_pair (per GPU: one conv's owned-row FLOPs / the slowest rank's conv "
                              "time; conv 1 also recomputes one halo plane per side)", "flops_per_launch": flops_gpu}
        kernel_stats = {"conv_ms_slowest_rank": conv_ms_max, "map_ms_slowest_rank": map_ms_max,
                        "conv_ms_this_rank": conv_ms, "map_ms_this_rank": map_ms}
        # every owned row against the single-GPU step of the whole shell, run on each rank's GPU
        r = runner.check_against_single_gpu(w1, w2)
        rel = torch.tensor([r["max_abs"] / max(r["max_ref"], 1e-30)], device=dev, dtype=torch.float64)
        dist.all_reduce(rel, op=dist.ReduceOp.MAX)
        cnt = torch.tensor([r["rows_checked"], r["rows_bit_exact"]], device=dev, dtype=torch.int64)
        dist.all_reduce(cnt)
        mrel = float(rel.item())
        parity = {"vs": "the single-GPU step (map, conv, conv) of the whole shell, on each rank's GPU",
                  "rows_checked": int(cnt[0].item()), "rows_bit_exact": int(cnt[1].item()),
                  "bit_exact": bool(int(cnt[1].item()) == int(cnt[0].item())), "max_rel": mrel, "tol": 1e-2,
                  "ok": bool(mrel < 1e-2 and int(cnt[0].item()) == n_total),
                  "note": "slab-local rows sum each row's 27 taps in another order (axes relabelled to put z "
                          "first), so bf16 outputs may differ by an ulp"}

    # ---- end to end through the host-buffer C-ABI call (pinned host in, host out)
    e2e = None
    if world == 1 and not args.no_e2e:
        feats_h = torch.empty((n_total, CI), dtype=torch.bfloat16).pin_memory()
        feats_h.copy_(feats.cpu())
        coords_h = torch.from_numpy(coords_np).pin_memory()
        out_h = torch.empty((n_total, CO), dtype=torch.bfloat16).pin_memory()
        layers = [(w1, None, "silu"), (w2, None, "none")]
        fe = feats_h.view(torch.int16).numpy()
        oh = out_h.view(torch.int16).numpy()
        ch = coords_h.numpy()
        for _ in range(2):
            ops.submconv_stack_host(ch, fe, layers, torch.bfloat16, torch.bfloat16, out=oh, device=dev)
        k_e2e = max(3, min(args.steps, 10))
        t0 = time.perf_counter()
        for _ in range(k_e2e):
            ops.submconv_stack_host(ch, fe, layers, torch.bfloat16, torch.bfloat16, out=oh, device=dev)
        dt = (time.perf_counter() - t0) / k_e2e
        e2e = {"value": n_total / dt, "unit": "voxels/s",
               "h2d_bytes_per_step": int(coords_h.numel() * 4 + feats_h.numel() * 2),
               "d2h_bytes_per_step": int(out_h.numel() * 2), "steps": k_e2e, "ms_per_step": dt * 1e3,
               "call": "tb_submconv_stack_host"}

    if world > 1 and not args.no_e2e:
        # end to end per rank: this rank's local coordinates and owned features from pinned host
        # memory, the halo exchange beside the slab's map, both convs, owned output rows back
        rows_np = runner.rows.cpu().numpy()
        coords_loc_h = torch.from_numpy(np.ascontiguousarray(coords_np[rows_np])).pin_memory()
        feats_own_h = runner.feats[runner.owned].cpu().pin_memory()
        out_own_h = torch.empty((runner.n_owned, CO), dtype=torch.bfloat16).pin_memory()
        coords_loc_d = torch.empty(coords_loc_h.shape, dtype=torch.int32, device=dev)

        def e2e_step():
            coords_loc_d.copy_(coords_loc_h, non_blocking=True)
            runner.feats[runner.owned].copy_(feats_own_h, non_blocking=True)
            runner.dist.load_coords(coords_loc_d)
            runner.step(w1, w2)
            out_own_h.copy_(runner.out[runner.owned], non_blocking=True)
        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        dist.barrier()
        k_e2e = max(3, min(args.steps, 10))
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k_e2e):
            e2e_step()
        b.record()
        torch.cuda.synchronize()
        te = torch.tensor([a.elapsed_time(b) / k_e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
        nb = torch.tensor([coords_loc_h.numel() * 4 + feats_own_h.numel() * 2, out_own_h.numel() * 2],
                          device=dev, dtype=torch.int64)
        dist.all_reduce(nb)
        e2e_ms = float(te.item())
        e2e = {"value": n_total / (e2e_ms / 1e3), "unit": "voxels/s", "h2d_bytes_per_step": int(nb[0].item()),
               "d2h_bytes_per_step": int(nb[1].item()), "steps": k_e2e, "ms_per_step": e2e_ms,
               "call": "per rank: pinned H2D of local coords + owned features, tb_dist_load_coords, "
                       "tb_dist_exchange + tb_dist_build_map, tb_dist_submconv_grow x2, D2H of owned rows "
                       "(CUDA events, slowest rank)"}

    if world > 1:
        # the z-slab partition runs once per voxel set (a decoder stage), outside the timed step:
        # timed here on a communicator-free dist of this rank (cut, local rows, one read-back),
        # slowest rank; -1 if it failed, so that every rank still takes the reduction below
        part_ms = -1.0
        try:
            pd = ops.Dist(dev, rank, world, halo_planes=runner.halo_planes)
            cg = runner.coords_global
            pd.partition(cg)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(3):
                pd.partition(cg)
            torch.cuda.synchronize()
            part_ms = (time.perf_counter() - t0) / 3 * 1e3
            pd.close()
        except Exception as ex:  # reported, never fatal: the step's numbers stand without it
            kernel_stats["partition_error"] = str(ex)[:200]
        tp = torch.tensor([part_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(tp, op=dist.ReduceOp.MAX)
        kernel_stats["partition_ms_slowest_rank"] = float(tp.item())
        kernel_stats["partition_note"] = ("tb_dist_partition_zslab, once per voxel set, outside the timed step "
                                          "(host wall clock around the call, which reads back the cut)")

    cpu_baseline = None
    if rank == 0 and not args.no_cpu:
        feats_c, wt1, wt2, nbr_c = _cpu_inputs(coords_np)
        nthreads = os.cpu_count() or 1
        sample = min(n_total, 1 << 18)
        spv, t_map, t_conv = cpu_reference_step(coords_np, nbr_c, feats_c, wt1, wt2, sample, nthreads)
        cpu_baseline = {"value": 1.0 / spv, "unit": "voxels/s", "cores": nthreads, "kind": "port",
                        "sample": f"full single-threaded neighbor map ({n_total} voxels, {t_map:.2f} s; "
                                  f"{_map_kind()}) + both fp32 convs (oracle port) on {sample} rows with "
                                  f"{nthreads} threads ({t_conv:.2f} s); per-voxel times summed"}
    if world > 1:
        dist.barrier()              # the other ranks wait while rank 0 times the CPU baseline

    launches_per_step = ops.NBR_MAP_LAUNCHES + 2   # neighbor map, conv, conv
    if world > 1:
        launches_per_step = runner.launches_per_step
    if rank == 0:
        clocks = sampler.summary()
        line = {
            "metric": METRIC, "value": value, "unit": "voxels/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (seeded noisy shell, random N(0,1) features, N(0,1/(27*64)) weights)",
            "config": {"workload": "c4: res-1024 noisy shell, neighbor map + conv(SiLU) + conv, C=64 bf16, "
                                   "fp32 accumulate", "voxels": n_total, "voxels_per_gpu": n_local,
                       "valid_pairs": pairs_total, "mean_valid_taps": pairs_total / n_total,
                       "parallelism": f"zslab{world}" if world > 1 else "single",
                       "issue": "one CUDA graph replay per rank per step" if world > 1 else "eager launches",
                       "l2": "inputs larger than L2 (features 625 MB, map 527 MB per step)"},
            "effective_tflops": eff_tflops,
            "dense27_equiv_tflops": 2 * 2.0 * 27 * CI * CO * n_total / (ms_step / 1e3) / 1e12,
            "roofline": roofline, "cpu_baseline": cpu_baseline, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps, "clocks": clocks, "kernels": kernel_stats,
        }
        if parity is not None:
            line["parity"] = parity
        if world == 1 and not args.no_configs:
            # every other BASELINE configuration, timed after the headline (not part of its value)
            line["configs"] = run_configs(dev, max(3, min(args.steps, 20)), max(3, args.warmup),
                                          cpu=not args.no_cpu)
        _emit(line)
    if world > 1:
        runner.close()
        dist.destroy_process_group()
    return 0


# ----------------------------------------------------------------------------- ConvNeXt block
CNX_METRIC = ("voxels/s through one sparse ConvNeXt block (3^3 conv + LayerNorm + Linear C->4C + SiLU + "
              "Linear 4C->C + residual), ~4.9M voxels C=64 (config 4 shell)")


def cpu_convnext_step(nbr_full, feats, cw, cb, nw, nb, w1, b1, w2, b2, sample, nthreads):
    """The block on `sample` output rows with the oracle port (C conv, numpy tail); s/voxel."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    n = feats.shape[0]
    row0 = (n - sample) // 2
    t0 = time.perf_counter()
    h = oracle.submconv_f32_mt_range(nbr_full, feats, oracle.weight_tap_major(cw), row0, sample, bias=cb,
                                     nthreads=nthreads)
    h = h[row0:row0 + sample] if h.shape[0] == n else h
    y = oracle.layer_norm(h, nw, nb)
    a = oracle.silu(y @ w1.T + b1)
    out = a @ w2.T + b2 + feats[row0:row0 + sample]
    dt = time.perf_counter() - t0
    assert out.shape == (sample, feats.shape[1])
    return dt / sample, dt


def run_convnext(args):
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _load_package()
    from trellis_cpp_b200 import ops, synth

    c = CI
    coords_np = synth.coords_for(args.workload)
    n = coords_np.shape[0]
    g = torch.Generator(device=dev).manual_seed(4321)
    bf = torch.bfloat16
    feats = torch.randn((n, c), device=dev, generator=g).to(bf)
    cw = (torch.randn((c, 27, c), device=dev, generator=g) / np.sqrt(27 * c)).to(bf)
    cb = 0.1 * torch.randn(c, device=dev, generator=g)
    nw = 1 + 0.1 * torch.randn(c, device=dev, generator=g)
    nb = 0.1 * torch.randn(c, device=dev, generator=g)
    w1 = (torch.randn((4 * c, c), device=dev, generator=g) / np.sqrt(c)).to(bf)
    b1 = 0.1 * torch.randn(4 * c, device=dev, generator=g)
    w2 = (torch.randn((c, 4 * c), device=dev, generator=g) / np.sqrt(4 * c)).to(bf)
    b2 = 0.1 * torch.randn(c, device=dev, generator=g)
    nbr = ops.build_neighbor_table(torch.from_numpy(coords_np).to(dev))
    h = torch.empty((n, c), dtype=torch.float32, device=dev)
    out = torch.empty((n, c), dtype=bf, device=dev)
    events = []

    def step(record=False):
        # the two launches of tb_sparse_convnext: conv (fp32 h), then the tail
        if record:
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record()
        ops.sparse_submconv(feats, nbr, cw, cb, out=h)
        if record:
            e[1].record()
        ops.convnext_tail(h, feats, nw, nb, w1, b1, w2, b2, out=out)
        if record:
            e[2].record()
            events.append(e)

    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    pairs = ops.count_valid_pairs(nbr, n)
    ops.check_device()
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    sampler.start()
    time.sleep(0.8)
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step(record=True)
    t1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ops.check_device()
    ms_step = t0.elapsed_time(t1) / args.steps
    conv_ms = float(np.mean([a.elapsed_time(b) for a, b, _ in events]))
    tail_ms = float(np.mean([b.elapsed_time(e) for _, b, e in events]))
    peak_tf, peak_bw, peak_kind = _peaks()
    tail_bytes = n * c * (4 + 2 + 2) + 2 * (4 * c * c) * 2     # h f32 + x + out bf16, weights
    tail_flops = 2.0 * 2 * 4 * c * c * n
    achieved = tail_bytes / (tail_ms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak_bw, "unit": "GB/s", "frac": achieved / peak_bw,
                "traffic": _profile_traffic("convnext_tail_c4.md"), "peak_source": f"{peak_kind} hbm_gbs",
                "kernel": "k_convnext_tail", "bytes_per_launch": tail_bytes,
                "tail_tflops": tail_flops / (tail_ms / 1e3) / 1e12}
    cpu = None
    if not args.no_cpu:
        rng = np.random.default_rng(3)
        f_np = rng.standard_normal((n, c)).astype(np.float32)
        mk = lambda *shape, s=1.0: (rng.standard_normal(shape) * s).astype(np.float32)  # noqa: E731
        sample = min(n, 1 << 16)
        nthreads = os.cpu_count() or 1
        spv, dt = cpu_convnext_step(nbr.cpu().numpy(), f_np, mk(c, 27, c, s=1 / np.sqrt(27 * c)), mk(c, s=0.1),
                                    1 + mk(c, s=0.1), mk(c, s=0.1), mk(4 * c, c, s=1 / np.sqrt(c)), mk(4 * c, s=0.1),
                                    mk(c, 4 * c, s=1 / np.sqrt(4 * c)), mk(c, s=0.1), sample, nthreads)
        cpu = {"value": 1.0 / spv, "unit": "voxels/s", "cores": nthreads, "kind": "port",
               "sample": f"oracle port: fp32 conv ({nthreads} threads) + numpy LayerNorm/MLP on {sample} rows "
                         f"({dt:.2f} s)"}
    line = {
        "metric": CNX_METRIC, "value": n / (ms_step / 1e3), "unit": "voxels/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded noisy shell, random N(0,1) features, random weights of the block's shapes)",
        "config": {"workload": f"{args.workload}: res-1024 noisy shell, ConvNeXt block C=64 bf16 operands, "
                               "fp32 h and accumulate, neighbor map prebuilt", "voxels": n, "valid_pairs": pairs,
                   "l2": "inputs larger than L2 (h 1.25 GB per step)"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": None,
        "gpu_launches": 2 * args.steps, "clocks": sampler.summary(),
        "kernels": {"conv_ms": conv_ms, "tail_ms": tail_ms,
                    "conv_tflops": 2.0 * c * c * pairs / (conv_ms / 1e3) / 1e12},
    }
    _emit(line)
    return 0


# ----------------------------------------------------------------------------- C2S up-block
C2S_METRIC = ("children/s through one SparseResBlockC2S3d up-block (norm1+SiLU, conv1 Cin->8*Cout, subdivide, "
              "channel-to-spatial + norm2 + SiLU, child map, conv2, skip), config-3 shell Cin=256 Cout=128")


def cpu_c2s_step(coords, mask, feats, w, cout, planes=4):
    """The oracle block on the parents of `planes` x-planes of the shell; seconds per child."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    xs = coords[:, -3]
    x0 = int(np.median(xs))
    sel = (xs >= x0) & (xs < x0 + planes)
    c = np.ascontiguousarray(coords[sel][:, -3:])
    t0 = time.perf_counter()
    out, child, _ = oracle.c2s_block(c, feats[sel], w, cout, ext_mask=mask[sel])
    dt = time.perf_counter() - t0
    return dt / max(1, child.shape[0]), dt, int(sel.sum()), int(child.shape[0])


def measure_c2s(dev, steps, warmup, cpu=True):
    """One tb_sparse_c2s call on config 3's shape, timed by CUDA events; returns a dict with the
    line's fields (value in children/s, roofline of conv1, CPU baseline)."""
    import torch
    from trellis_cpp_b200 import ops, synth

    cin, cout = 256, 128
    parents = synth.coords_for("c3")
    mask_np = synth.c3_mask(parents)
    n = parents.shape[0]
    rng = np.random.default_rng(33)
    bf = torch.bfloat16

    def t(a, dt=torch.float32):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev).to(dt)
    w = {
        "norm1.weight": (1 + 0.1 * rng.standard_normal(cin)).astype(np.float32),
        "norm1.bias": (0.1 * rng.standard_normal(cin)).astype(np.float32),
        "conv1.weight": (rng.standard_normal((8 * cout, 27, cin)) / np.sqrt(27 * cin)).astype(np.float32),
        "conv1.bias": (0.1 * rng.standard_normal(8 * cout)).astype(np.float32),
        "conv2.weight": (rng.standard_normal((cout, 27, cout)) / np.sqrt(27 * cout)).astype(np.float32),
        "conv2.bias": (0.1 * rng.standard_normal(cout)).astype(np.float32),
    }
    feats_np = rng.standard_normal((n, cin)).astype(np.float32)
    prm = {k: t(v, bf if k.endswith("conv1.weight") or k.endswith("conv2.weight") else torch.float32)
           for k, v in w.items()}
    coords = torch.from_numpy(parents).to(dev)
    feats = t(feats_np, bf)
    mask = torch.from_numpy(mask_np).to(dev)
    m_children = int(mask_np.sum())

    def step():
        return ops.sparse_c2s(coords, feats, prm, cout, ext_mask=mask, max_children=m_children)

    for _ in range(max(3, warmup)):
        out, child, _ = step()
    torch.cuda.synchronize()
    ops.check_device()
    m = child.shape[0]
    ms_step = _time_op(step, steps, 0)
    ops.check_device()

    # conv1 alone (the block's dominant kernel) for the roofline
    nbr = ops.build_neighbor_table(coords)
    h = torch.empty((n, cin), dtype=bf, device=dev)
    h.copy_(feats)
    h1 = torch.empty((n, 8 * cout), dtype=torch.float32, device=dev)
    conv1_ms = _time_op(lambda: ops.sparse_submconv(h, nbr, prm["conv1.weight"], prm["conv1.bias"], out=h1), 10, 3)
    pairs = ops.count_valid_pairs(nbr, n)
    peak_tf, peak_bw, peak_kind = _peaks()
    flops1 = 2.0 * cin * 8 * cout * pairs
    achieved = flops1 / (conv1_ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                "traffic": None, "peak_source": f"{peak_kind} bf16_tflops (burst)", "kernel": "k_submconv_brick (conv1)",
                "flops_per_launch": flops1, "conv1_ms": conv1_ms}
    cpu_b = None
    if cpu:
        spc, dt, np_, nc_ = cpu_c2s_step(parents, mask_np, feats_np, w, cout)
        cpu_b = {"value": 1.0 / spc, "unit": "children/s", "cores": os.cpu_count() or 1, "kind": "port",
                 "cpu": _cpu_model(),
                 "sample": f"oracle port (numpy fp64) c2s_block on {np_} parents of 4 x-planes -> {nc_} children "
                           f"({dt:.2f} s)"}
    del h, h1, nbr
    torch.cuda.empty_cache()
    return {"workload": "c3: res-256 shell parents -> res-512 children, external (texture-decoder style) mask, "
                        "Cin=256 Cout=128 bf16 operands, fp32 conv outputs and skip",
            "metric": "children/s through one SparseResBlockC2S3d up-block",
            "value": m / (ms_step / 1e3), "unit": "children/s", "ms_per_step": ms_step, "steps": steps,
            "parents": n, "children": m, "parent_valid_pairs": pairs, "roofline": roofline, "cpu_baseline": cpu_b,
            "l2": "conv1 output 1.0 GB per step (larger than L2)",
            "launches_per_step": 2 * ops.NBR_MAP_LAUNCHES + 9}


def run_c2s(args):
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _load_package()
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    sampler.start()
    time.sleep(0.8)
    r = measure_c2s(dev, args.steps, args.warmup, cpu=not args.no_cpu)
    sampler.stop()
    line = {
        "metric": C2S_METRIC, "value": r["value"], "unit": "children/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": r["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded res-256 noisy shell, seeded thickness mask, random weights of the block's shapes)",
        "config": {"workload": r["workload"], "parents": r["parents"], "children": r["children"],
                   "parent_valid_pairs": r["parent_valid_pairs"], "l2": r["l2"]},
        "roofline": r["roofline"], "cpu_baseline": r["cpu_baseline"], "e2e": None,
        "gpu_launches": r["launches_per_step"] * args.steps, "clocks": sampler.summary(),
    }
    _emit(line)
    return 0


# ----------------------------------------------------------------------------- dual-grid mesh
MESH_METRIC = ("voxels/s through dual_grid_to_mesh (src/dual_grid.cpp:16-56): dual vertices, coordinate "
               "lookups of each intersected edge's quad, split and triangles in the reference's order")


def cpu_mesh_step(coords, f7, res):
    """The reference's own dual_grid_to_mesh (oracle/_ref) when it was built, else the oracle
    port; one call over the whole workload. Returns (seconds per voxel, seconds, kind, F)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    t0 = time.perf_counter()
    if oracle.ref_available():
        _, faces = oracle.ref_dual_grid_mesh(coords, f7, res)
        kind = "reference"
    else:
        _, faces, _ = oracle.dual_grid_mesh(coords, f7, res)
        kind = "port"
    dt = time.perf_counter() - t0
    return dt / len(coords), dt, kind, int(faces.shape[0])


def run_mesh(args):
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _load_package()
    from trellis_cpp_b200 import ops, synth

    coords_np = np.ascontiguousarray(synth.coords_for(args.workload)[:, -3:])
    n = coords_np.shape[0]
    res = 1024
    f7_np = (np.random.default_rng(77).standard_normal((n, 7)) * 2).astype(np.float32)
    coords = torch.from_numpy(coords_np).to(dev)
    f7 = torch.from_numpy(f7_np).to(dev)
    faces = None
    for _ in range(max(3, args.warmup)):
        _, faces = ops.dual_grid_mesh(coords, f7, res)
    torch.cuda.synchronize()
    ops.check_device()
    nf = faces.shape[0]
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    sampler.start()
    time.sleep(0.8)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        ops.dual_grid_mesh(coords, f7, res)
    e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ops.check_device()
    ms_step = e0.elapsed_time(e1) / args.steps

    # end to end: pinned host inputs up, the call, vertices and triangles down
    e2e = None
    if not args.no_e2e:
        hc = torch.from_numpy(coords_np).pin_memory()
        hf = torch.from_numpy(f7_np).pin_memory()
        hv = torch.empty((n, 3), dtype=torch.float32).pin_memory()
        hfa = torch.empty((6 * n, 3), dtype=torch.int32).pin_memory()
        dc = torch.empty_like(coords)
        df = torch.empty_like(f7)

        def e2e_step():
            dc.copy_(hc, non_blocking=True)
            df.copy_(hf, non_blocking=True)
            v, fa = ops.dual_grid_mesh(dc, df, res)
            hv.copy_(v, non_blocking=True)
            hfa[: fa.shape[0]].copy_(fa, non_blocking=True)
        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize()
        x0 = torch.cuda.Event(enable_timing=True)
        x1 = torch.cuda.Event(enable_timing=True)
        k = max(1, min(args.steps, 20))
        x0.record()
        for _ in range(k):
            e2e_step()
        x1.record()
        torch.cuda.synchronize()
        ms_e2e = x0.elapsed_time(x1) / k
        e2e = {"value": n / (ms_e2e / 1e3), "unit": "voxels/s", "h2d_bytes_per_step": n * 40,
               "d2h_bytes_per_step": n * 12 + nf * 12, "steps": k, "ms_per_step": ms_e2e,
               "call": "tb_dual_grid_mesh with pinned host inputs and outputs"}
    _, peak_bw, peak_kind = _peaks()
    alg_bytes = n * (12 + 28 + 12) + nf * 12
    achieved = alg_bytes / (ms_step / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak_bw, "unit": "GB/s", "frac": achieved / peak_bw,
                "traffic": None, "peak_source": f"{peak_kind} hbm_gbs",
                "kernel": "tb_dual_grid_mesh (whole call: seven-tap map build + k_mesh_count + scan + k_mesh_emit)",
                "bytes_per_launch": alg_bytes}
    cpu = None
    if not args.no_cpu:
        spv, dt, kind, cpu_f = cpu_mesh_step(coords_np, f7_np, res)
        if cpu_f != nf:
            raise RuntimeError(f"CPU and GPU triangle counts differ: {cpu_f} vs {nf}")
        cpu = {"value": 1.0 / spv, "unit": "voxels/s", "cores": 1, "kind": kind,
               "sample": ("the reference's own dual_grid_to_mesh (compiled from its sources)" if kind == "reference"
                          else "oracle port of dual_grid_to_mesh") + f", single-threaded, whole workload ({dt:.2f} s)"}
    line = {
        "metric": MESH_METRIC, "value": n / (ms_step / 1e3), "unit": "voxels/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded res-1024 noisy shell, decoder-head fields N(0, 2^2))",
        "config": {"workload": f"{args.workload}: res-1024 noisy shell as the decoded voxels, 7 fields per voxel",
                   "voxels": n, "triangles": nf,
                   "l2": f"inputs {n * 40 / 1e6:.0f} MB, outputs {(n * 12 + nf * 12) / 1e6:.0f} MB per step "
                         "(larger than L2)"},
        "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
        "gpu_launches": (ops.NBR_MAP_LAUNCHES + 3) * args.steps, "clocks": sampler.summary(),
    }
    _emit(line)
    return 0


# ----------------------------------------------------------------------------- decoder UNet
DEC_METRIC = ("output voxels/s through the sparse decoder UNet (from_latent, 4 stages of ConvNeXt blocks + C2S "
              "up-blocks, LayerNorm + output_layer), res-32 shell -> res 512")
DEC_STAGES = [(1024, 4, 512), (512, 16, 256), (256, 8, 128), (128, 4, 64)]    # C, ConvNeXt blocks, Cout


def _dec_inputs():
    from trellis_cpp_b200 import synth
    coords = synth.shell(32, 12.5, 1.0, 8.0, 11, 2.0)
    stage_coords, masks = [coords], []
    res, rad, amp, sp = 32, 12.5, 1.0, 8.0
    for _ in DEC_STAGES:
        m = synth.child_mask(stage_coords[-1], res, rad, amp, sp, 11, 0.5)
        masks.append(m)
        c = stage_coords[-1][:, -3:].astype(np.int64)
        idx = np.nonzero(m.reshape(-1))[0]
        i, o = idx // 8, idx % 8
        kids = np.stack([2 * c[i, 0] + (o & 1), 2 * c[i, 1] + ((o >> 1) & 1), 2 * c[i, 2] + ((o >> 2) & 1)], 1)
        stage_coords.append(np.concatenate([np.zeros((kids.shape[0], 1), np.int64), kids], 1).astype(np.int32))
        res, rad, amp, sp = 2 * res, 2 * rad, 2 * amp, 2 * sp
    return stage_coords, masks


def _dec_weights(rng_or_gen, make):
    w = {"from_latent.weight": make((1024, 32), 1 / np.sqrt(32), True), "from_latent.bias": make((1024,), 0.1, False)}
    for s, (c, nblk, cout) in enumerate(DEC_STAGES):
        for j in range(nblk):
            p = f"blocks.{s}.{j}."
            w.update({p + "conv.weight": make((c, 27, c), 1 / np.sqrt(27 * c), True), p + "conv.bias": make((c,), 0.1, False),
                      p + "norm.weight": make((c,), 0.1, False, 1.0), p + "norm.bias": make((c,), 0.1, False),
                      p + "mlp.0.weight": make((4 * c, c), 1 / np.sqrt(c), True), p + "mlp.0.bias": make((4 * c,), 0.1, False),
                      p + "mlp.2.weight": make((c, 4 * c), 1 / np.sqrt(4 * c), True), p + "mlp.2.bias": make((c,), 0.1, False)})
        p = f"blocks.{s}.{nblk}."
        w.update({p + "norm1.weight": make((c,), 0.1, False, 1.0), p + "norm1.bias": make((c,), 0.1, False),
                  p + "conv1.weight": make((8 * cout, 27, c), 1 / np.sqrt(27 * c), True),
                  p + "conv1.bias": make((8 * cout,), 0.1, False),
                  p + "conv2.weight": make((cout, 27, cout), 1 / np.sqrt(27 * cout), True),
                  p + "conv2.bias": make((cout,), 0.1, False)})
    w["output_layer.weight"] = make((7, 64), 1 / np.sqrt(64), True)
    w["output_layer.bias"] = make((7,), 0.1, False)
    return w


def _decode(ops, w, latent, coords, masks, stage_pairs=None):
    """decode_unet through the library's C-ABI ops (device tensors); returns (out7, coords).

    Each stage's map and ConvNeXt blocks run on the stage's rows in key order (tb_sort_rows), the
    order whose 128-row tiles the conv kernels read as contiguous neighbour ranges; the C2S
    block's children come parent-major, so the stage's rows are gathered into key order and the
    blocks' output is scattered back, and every output keeps the reference's row order."""
    import torch
    h = ops.linear(latent, w["from_latent.weight"], w["from_latent.bias"])
    for s, (c, nblk, cout) in enumerate(DEC_STAGES):
        perm = ops.sort_rows(coords)
        hs = ops.gather_rows(h, perm)
        nbr = ops.build_neighbor_table(ops.gather_rows(coords, perm))
        if stage_pairs is not None:
            stage_pairs.append(ops.count_valid_pairs(nbr, coords.shape[0]))
        for j in range(nblk):
            p = f"blocks.{s}.{j}."
            hs = ops.sparse_convnext(hs, nbr, w[p + "conv.weight"], w[p + "conv.bias"], w[p + "norm.weight"],
                                     w[p + "norm.bias"], w[p + "mlp.0.weight"], w[p + "mlp.0.bias"],
                                     w[p + "mlp.2.weight"], w[p + "mlp.2.bias"])
        h = ops.scatter_rows(torch.empty_like(h), perm, hs)
        p = f"blocks.{s}.{nblk}."
        prm = {k[len(p):]: v for k, v in w.items() if k.startswith(p)}
        h, coords, _ = ops.sparse_c2s(coords, h, prm, cout, ext_mask=masks[s], max_children=int(masks[s].sum()))
    y = ops.layer_norm(h, eps=1e-5)
    return ops.linear(y, w["output_layer.weight"], w["output_layer.bias"], out_dtype=torch.float32), coords


def cpu_decode_patch(stage0, nthreads, patch=2):
    """The decoder on the parents of a patch x, y in [x0, x0 + patch) of the res-32 shell with the
    oracle port: fp32 multi-threaded convs (orc_submconv_f32_mt), numpy LayerNorm / MLP / linears,
    the oracle's subdivide and gathers, shell-following masks as in the GPU run, random weights
    of the same shapes (the time does not depend on their values). Returns (s per output voxel,
    s, parents, output voxels)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from trellis_cpp_b200 import synth
    rng = np.random.default_rng(5)
    c = stage0[:, -3:]
    x0, y0 = int(np.median(c[:, 0])), int(np.median(c[:, 1]))
    par = stage0[(c[:, 0] >= x0) & (c[:, 0] < x0 + patch) & (c[:, 1] >= y0 - 4) & (c[:, 1] < y0 + 4)]
    coords = np.ascontiguousarray(par[:, -3:])

    def wt(co, ci):
        return oracle.weight_tap_major(rng.standard_normal((co, 27, ci), dtype=np.float32) / np.sqrt(27 * ci))
    t0 = time.perf_counter()
    h = rng.standard_normal((coords.shape[0], 32), dtype=np.float32) @ \
        (rng.standard_normal((32, 1024), dtype=np.float32) / np.sqrt(32))
    res, rad, amp, sp = 32, 12.5, 1.0, 8.0
    for c_in, nblk, cout in DEC_STAGES:
        nbr = oracle.build_neighbor_table(coords)
        for _ in range(nblk):
            conv = oracle.submconv_f32_mt(nbr, h, wt(c_in, c_in), nthreads=nthreads)
            y = oracle.layer_norm(conv).astype(np.float32)
            a = oracle.silu(y @ (rng.standard_normal((c_in, 4 * c_in), dtype=np.float32) / np.sqrt(c_in)))
            h = (a.astype(np.float32) @ (rng.standard_normal((4 * c_in, c_in), dtype=np.float32) / np.sqrt(4 * c_in))
                 + h).astype(np.float32)
        mask = synth.child_mask(coords, res, rad, amp, sp, 11, 0.5)
        hn = oracle.silu(oracle.layer_norm(h)).astype(np.float32)
        h1 = oracle.submconv_f32_mt(nbr, hn, wt(8 * cout, c_in), nthreads=nthreads)
        child, gidx, _ = oracle.subdivide(coords, mask)
        hc = oracle.silu(oracle.layer_norm(oracle.c2s_gather(h1, gidx, cout))).astype(np.float32)
        nbr2 = oracle.build_neighbor_table(child)
        h = oracle.submconv_f32_mt(nbr2, hc, wt(cout, cout), nthreads=nthreads) + \
            np.repeat(oracle.c2s_gather(h, gidx, c_in // 8), cout // (c_in // 8), axis=1)
        coords = np.ascontiguousarray(child)
        res, rad, amp, sp = 2 * res, 2 * rad, 2 * amp, 2 * sp
    out = oracle.layer_norm(h, eps=1e-5) @ rng.standard_normal((64, 7))
    dt = time.perf_counter() - t0
    return dt / max(1, out.shape[0]), dt, par.shape[0], out.shape[0]


def run_decode(args):
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _load_package()
    from trellis_cpp_b200 import ops
    stage_coords, masks_np = _dec_inputs()
    g = torch.Generator(device=dev).manual_seed(77)

    def make(shape, scale, weight, offset=0.0):
        t = offset + scale * torch.randn(shape, device=dev, generator=g)
        return t.bfloat16() if weight else t.float()
    w = _dec_weights(g, make)
    coords = torch.from_numpy(stage_coords[0]).to(dev)
    masks = [torch.from_numpy(m).to(dev) for m in masks_np]
    latent = torch.randn((coords.shape[0], 32), device=dev, generator=g).bfloat16()
    pairs = []
    out, final = _decode(ops, w, latent, coords, masks, pairs)
    for _ in range(max(2, args.warmup - 1)):
        _decode(ops, w, latent, coords, masks)
    torch.cuda.synchronize()
    ops.check_device()
    m_final = final.shape[0]
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    sampler.start()
    time.sleep(0.8)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        _decode(ops, w, latent, coords, masks)
    e1.record()
    torch.cuda.synchronize()
    sampler.stop()
    ops.check_device()
    ms = e0.elapsed_time(e1) / args.steps
    # algorithmic FLOPs: convs on present pairs, MLPs and linears per voxel
    ns = [sc.shape[0] for sc in stage_coords]
    flops = 2.0 * 32 * 1024 * ns[0] + 2.0 * 64 * 7 * ns[-1]
    child_pairs = []
    for s, (c, nblk, cout) in enumerate(DEC_STAGES):
        flops += nblk * (2.0 * c * c * pairs[s] + 2 * 2.0 * 4 * c * c * ns[s])
        flops += 2.0 * c * 8 * cout * pairs[s]
        nb_child = ops.build_neighbor_table(torch.from_numpy(stage_coords[s + 1]).to(dev))
        child_pairs.append(ops.count_valid_pairs(nb_child, ns[s + 1]))
        flops += 2.0 * cout * cout * child_pairs[-1]
    peak_tf, _, peak_kind = _peaks()
    achieved = flops / (ms / 1e3) / 1e12
    roofline = {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s", "frac": achieved / peak_tf,
                "traffic": None, "peak_source": f"{peak_kind} bf16_tflops (burst)",
                "kernel": "the whole decode (convs, MLPs, linears)", "flops_per_step": flops}
    line = {
        "metric": DEC_METRIC, "value": m_final / (ms / 1e3), "unit": "voxels/s", "n_gpus": 1, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded res-32 noisy shell, seeded shell-following masks, random weights of the "
                "reference's stage shapes)",
        "config": {"workload": "decode_unet, stage table 1024x4/512x16/256x8/128x4 + C2S, out 7 channels",
                   "voxels_per_stage": ns, "parent_pairs": pairs, "child_pairs": child_pairs,
                   "l2": "weights 0.9 GB and activations larger than L2"},
        "roofline": roofline, "cpu_baseline": None, "e2e": None, "clocks": sampler.summary(),
    }
    if not args.no_cpu:
        nthreads = os.cpu_count() or 1
        spv, dt, npar, nout = cpu_decode_patch(stage_coords[0], nthreads)
        line["cpu_baseline"] = {"value": 1.0 / spv, "unit": "voxels/s", "cores": nthreads, "kind": "port",
                                "sample": f"oracle port (fp32 multi-threaded convs, numpy MLPs, the oracle's "
                                          f"subdivide and gathers) on a {npar}-parent patch of the shell grown to "
                                          f"{nout} output voxels ({dt:.1f} s)"}
    _emit(line)
    return 0


# ----------------------------------------------------------------------------- every BASELINE config
# One timed entry per configuration of BASELINE.json (C1, C2, C3, C5 at C=32 and C=512; C4 is the
# headline line itself) plus two row-order probes of the C4 conv. Each entry: the conv (or block)
# timed with CUDA events on HBM-resident inputs, its roofline against the measured peak, a parity
# check of sampled rows against the oracle, and the oracle port timed on a bounded sample.
CFG_TABLE = {
    # name: (coords, ci, co, dtype, epilogue, cpu sample rows, bias std)
    "c1": ("c1", 64, 64, "f32", "none", None, 0.0),
    "c2": ("c2", 256, 256, "f16", "none", 4096, 0.01),
    "c5_32": ("c5_32", 32, 32, "f16", "none", 65536, 0.0),
    "c5_512": ("c5_512", 512, 512, "f16", "none", 1024, 0.0),
}


def _l2_flush_buffer(dev):
    import torch
    return torch.empty(64 << 20, dtype=torch.float32, device=dev)     # 256 MB > the 126 MB L2


def _time_op(fn, steps, warmup, flush=None):
    """Mean ms per call of fn() by CUDA events on the current stream. With `flush` (a buffer
    larger than L2) the buffer is rewritten before every timed call, outside the events."""
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if flush is None:
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps
    evs = []
    for _ in range(steps):
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        evs.append((a, b))
    torch.cuda.synchronize()
    return float(np.mean([a.elapsed_time(b) for a, b in evs]))


def _sample_rows(n, k, seed):
    rng = np.random.default_rng(seed)
    return np.sort(rng.choice(n, size=min(n, k), replace=False)).astype(np.int64)


def _torch_conv_rows(nbr, feats, w, bias, n, rows, silu):
    """Output rows `rows` of the conv as a plain torch fp32 gather + matmul on the device (an
    independent check of the kernel's arithmetic; absent taps contribute zero)."""
    import torch
    r = torch.from_numpy(np.ascontiguousarray(rows, dtype=np.int64)).to(feats.device)
    nb = nbr.view(27, n)[:, r].long()                                     # [27, m]
    present = (nb != n).unsqueeze(-1)
    x = feats.float()[nb.clamp(max=n - 1)] * present                     # [27, m, ci]
    y = torch.einsum("tmc,otc->mo", x, w.float())
    if bias is not None:
        y = y + bias.float()
    return torch.nn.functional.silu(y) if silu else y


def _mini_problem(nbr, feats, n, rows):
    """The conv of output rows `rows` as a small stand-alone problem for the CPU: the rows come
    first in the local order, followed by every other row they read. Returns (tap-major int32 map
    [27 * n_loc] with sentinel n_loc, float32 features [n_loc, ci]); local rows 0..len(rows)-1
    are the requested ones. Only these rows leave the device."""
    import torch
    r_t = torch.from_numpy(np.ascontiguousarray(rows, dtype=np.int64)).to(feats.device)
    nb = nbr.view(27, n)[:, r_t].cpu().numpy().astype(np.int64)        # [27, m]
    m = rows.size
    present = nb != n
    others = np.setdiff1d(np.unique(nb[present]), rows)
    order = np.concatenate([np.asarray(rows, dtype=np.int64), others])
    perm = np.argsort(order, kind="stable")
    sorted_ids = order[perm]
    n_loc = order.size
    loc = np.full((27, n_loc), n_loc, dtype=np.int32)
    loc[:, :m] = np.where(present, perm[np.searchsorted(sorted_ids, np.where(present, nb, sorted_ids[0]))], n_loc)
    f = feats[torch.from_numpy(order).to(feats.device)].float().cpu().numpy()
    return np.ascontiguousarray(loc.reshape(-1)), f


def measure_conv_config(name, dev, steps, warmup, cpu=True, coords_np=None, order_note=None):
    """One BASELINE conv configuration: map prebuilt, one conv timed; returns the entry dict."""
    import torch
    from trellis_cpp_b200 import ops, synth
    cname, ci, co, dts, epi, cpu_rows, bstd = CFG_TABLE[name]
    if coords_np is None:
        coords_np = synth.coords_for(cname)
    n = coords_np.shape[0]
    tdt = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}[dts]
    g = torch.Generator(device=dev).manual_seed(zlib.crc32(name.encode()) & 0xFFFF)
    feats = torch.randn((n, ci), device=dev, generator=g).to(tdt)
    w = (torch.randn((co, 27, ci), device=dev, generator=g) / np.sqrt(27 * ci)).to(tdt)
    bias = (bstd * torch.randn(co, device=dev, generator=g)) if bstd else None
    coords = torch.from_numpy(coords_np).to(dev)
    nbr = torch.empty(27 * n, dtype=torch.int32, device=dev)
    ops.build_neighbor_table(coords, out=nbr)
    out = torch.empty((n, co), dtype=tdt, device=dev)
    small = n * ci * feats.element_size() + 108 * n < (256 << 20)
    flush = _l2_flush_buffer(dev) if small else None
    conv = lambda: ops.sparse_submconv(feats, nbr, w, bias, epi=epi, out=out)   # noqa: E731
    conv_ms = _time_op(conv, steps, warmup, flush)
    map_ms = _time_op(lambda: ops.build_neighbor_table(coords, out=nbr), max(3, steps // 2), 2, flush)
    ops.check_device()
    pairs = ops.count_valid_pairs(nbr, n)
    peak_tf, peak_bw, peak_kind = _peaks()
    esz = feats.element_size()
    flops = 2.0 * ci * co * pairs
    bytes_ = n * (ci + co) * esz + 108 * n + 27 * ci * co * esz + (4 * co if bias is not None else 0)
    t_tensor = flops / (peak_tf * 1e12) if dts != "f32" else 0.0
    t_hbm = bytes_ / (peak_bw * 1e9)
    if dts == "f32" or t_hbm >= t_tensor:
        achieved = bytes_ / (conv_ms / 1e3) / 1e9
        roof = {"bound": "hbm", "achieved": achieved, "peak": peak_bw, "unit": "GB/s", "frac": achieved / peak_bw,
                "peak_source": f"{peak_kind} hbm_gbs", "bytes_per_launch": bytes_}
    else:
        achieved = flops / (conv_ms / 1e3) / 1e12
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak_tf, "unit": "TFLOP/s",
                "frac": achieved / peak_tf, "peak_source": f"{peak_kind} bf16_tflops (burst)",
                "flops_per_launch": flops}
    path = "k_conv_f32 (FFMA)" if dts == "f32" else (
        "k_submconv_pair" if ci in (32, 64) and co in (32, 64) else
        ("k_submconv_brick" if ci % 64 == 0 else "k_submconv_tc (gather4)"))
    roof["kernel"] = path
    # parity of sampled rows against a plain torch fp32 gather + matmul of the same operands
    rows = _sample_rows(n, 256, 5)
    ref = _torch_conv_rows(nbr, feats, w, bias, n, rows, epi == "silu")
    got = out[torch.from_numpy(rows).to(dev)].float()
    mrel = float((got - ref).abs().max() / ref.abs().max().clamp_min(1e-30))
    w_h = w.float().cpu().numpy()
    tol = 1e-4 if dts == "f32" else 1e-2
    entry = {
        "workload": synth.CONFIGS[cname]["desc"] if order_note is None else order_note, "voxels": n,
        "ci": ci, "co": co, "dtype": dts, "metric": "voxels/s through one 3^3 submanifold conv (map prebuilt)",
        "value": n / (conv_ms / 1e3), "unit": "voxels/s", "ms_per_step": conv_ms, "steps": steps,
        "map_ms": map_ms, "valid_pairs": pairs, "mean_valid_taps": pairs / max(n, 1),
        "effective_tflops": flops / (conv_ms / 1e3) / 1e12, "roofline": roof,
        "l2": "L2 flushed before each timed call (inputs under 256 MB)" if small else "inputs larger than L2",
        "parity": {"vs": "torch fp32 gather + matmul of the same operands", "rows_checked": int(rows.size),
                   "max_rel": mrel,
                   "tol": tol, "ok": mrel < tol},
    }
    if cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle      # the CPU baseline leg: the oracle port is what is timed here
        nthreads = os.cpu_count() or 1
        sample = n if cpu_rows is None else min(n, cpu_rows)
        row0 = (n - sample) // 2
        nbr_s, f_s = _mini_problem(nbr, feats, n, np.arange(row0, row0 + sample, dtype=np.int64))
        wt = oracle.weight_tap_major(w_h)
        t0 = time.perf_counter()
        oracle.submconv_f32_mt_range(nbr_s, f_s, wt, 0, sample, nthreads=nthreads)
        dt = time.perf_counter() - t0
        entry["cpu_baseline"] = {"value": sample / dt, "unit": "voxels/s", "cores": nthreads, "kind": "port",
                                 "cpu": _cpu_model(),
                                 "sample": f"oracle port fp32 conv on {sample} consecutive rows (their neighbor rows "
                                           f"gathered first), {nthreads} threads ({dt:.2f} s)"}
    del feats, w, nbr, out, flush
    torch.cuda.empty_cache()
    return entry


def _c4_orders(dev):
    """The C4 conv's input in two other row orders than the generator's x-major one:
    (a) the order a decoder produces it -- the res-512 (half-scale) shell subdivided with a seeded
    thickness mask into res-1024 children by tb_subdivide, parent-major and octant-ascending
    (src/sparse.cpp:205-222); (b) the C4 voxels in Morton (z-order curve) order."""
    import torch
    from trellis_cpp_b200 import ops, synth
    parents = synth.coords_for("c4s")
    mask = synth.child_mask(parents, 512, 220.0, 8.0, 64.0, 4, 0.5)
    child, _, _ = ops.subdivide(torch.from_numpy(parents).to(dev), torch.from_numpy(mask.reshape(-1)).to(dev),
                                int(mask.sum()))
    child = child.cpu().numpy()
    c4 = synth.coords_for("c4")

    def morton(c):
        def spread(v):
            v = v.astype(np.uint64) & np.uint64(0x1FFFFF)
            r = np.zeros_like(v)
            for b in range(21):
                r |= ((v >> np.uint64(b)) & np.uint64(1)) << np.uint64(3 * b)
            return r
        return spread(c[:, -3]) << np.uint64(2) | spread(c[:, -2]) << np.uint64(1) | spread(c[:, -1])
    c4m = np.ascontiguousarray(c4[np.argsort(morton(c4), kind="stable")])
    xsorted = np.ascontiguousarray(child[np.lexsort((child[:, -1], child[:, -2], child[:, -3]))])
    return np.ascontiguousarray(child), xsorted, c4m


def run_configs_line(args):
    """`--op configs`: the per-config entries alone, as one JSON line."""
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _load_package()
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    sampler.start()
    time.sleep(0.8)
    res = run_configs(dev, max(3, min(args.steps, 20)), max(3, args.warmup), cpu=not args.no_cpu)
    sampler.stop()
    _emit({"metric": "per-configuration conv throughput (BASELINE configs C1-C5)", "n_gpus": 1,
           "configs": res, "clocks": sampler.summary()})
    return 0


def run_one_config(args):
    """`--op config --config NAME`: one BASELINE configuration's conv alone (for profiling)."""
    import torch
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    _load_package()
    if args.config == "c3":
        r = measure_c2s(dev, max(3, args.steps), max(3, args.warmup), cpu=not args.no_cpu)
    else:
        r = measure_conv_config(args.config, dev, max(3, args.steps), max(3, args.warmup), cpu=not args.no_cpu)
    _emit({"metric": f"configuration {args.config}", "n_gpus": 1, "configs": {args.config: r}})
    return 0


def run_configs(dev, steps, warmup, cpu=True):
    """Every BASELINE configuration other than the headline C4 step (see CFG_TABLE), C3's C2S
    block, and the C4 conv on decoder-ordered and Morton-ordered rows."""
    import torch
    res = {}
    for name in ("c1", "c2", "c5_32", "c5_512"):
        st = steps if name != "c5_512" else max(3, steps // 4)
        res[name] = measure_conv_config(name, dev, st, warmup, cpu)
    res["c3"] = measure_c2s(dev, max(3, steps // 2), warmup, cpu)
    dec, dec_sorted, c4m = _c4_orders(dev)
    CFG_TABLE["c4_order"] = ("c4", 64, 64, "bf16", "silu", None, 0.0)
    res["c4_decoder_order"] = measure_conv_config(
        "c4_order", dev, steps, warmup, False, dec,
        "res-512 shell subdivided to res 1024 (decoder order: parent-major, octant-ascending), C=64 bf16")
    res["c4_decoder_sorted"] = measure_conv_config(
        "c4_order", dev, steps, warmup, False, dec_sorted,
        "the same children sorted x-major (the reference's key order), C=64 bf16")
    res["c4_morton"] = measure_conv_config(
        "c4_order", dev, steps, warmup, False, c4m, "C4 shell in Morton order, C=64 bf16")
    res["c4_xmajor"] = measure_conv_config(
        "c4_order", dev, steps, warmup, False, None, "C4 shell in x-major order (as the headline), C=64 bf16")
    torch.cuda.empty_cache()
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end leg")
    ap.add_argument("--workload", default=WORKLOAD, choices=["c4", "c4s"],
                    help="c4 (default, the benchmark) or c4s (half scale, for profiler captures)")
    ap.add_argument("--no-configs", action="store_true", help="skip the per-config entries of the headline line")
    ap.add_argument("--config", default="c2", choices=["c1", "c2", "c3", "c5_32", "c5_512"],
                    help="the configuration of --op config")
    ap.add_argument("--op", default="stack", choices=["stack", "convnext", "c2s", "decode", "mesh", "configs", "config"],
                    help="stack (default, the benchmark: map + conv x2), convnext (one ConvNeXt block), c2s "
                         "(one C2S up-block), decode (the sparse decoder UNet) or mesh (dual_grid_to_mesh)")
    args = ap.parse_args()
    if args.op in ("convnext", "c2s", "decode", "mesh", "configs", "config"):
        if args.impl == "reference" or args.gpus != 1:
            print(json.dumps({"impl": args.impl, "unavailable": f"--op {args.op} is a single-GPU measurement of "
                              "our kernels; its CPU baseline is in the line's cpu_baseline"}))
            return 0
        return {"convnext": run_convnext, "c2s": run_c2s, "decode": run_decode, "mesh": run_mesh,
                "configs": run_configs_line, "config": run_one_config}[args.op](args)
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
