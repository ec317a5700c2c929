"""The reference arm of bench.py runs on the host cores only, so its output contract is checked
here without a GPU: one JSON line with the headline metric, a cpu_baseline naming its kind, cores
and sample, and an e2e entry with no host-device bytes; the other ranks of a torchrun launch exit
0 without work, and the single-GPU measurement ops answer with an `unavailable` line."""
import json
import os
import subprocess
import sys

from conftest import ROOT

BENCH = os.path.join(ROOT, "bench.py")


def _run(args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, BENCH] + args, capture_output=True, text=True, env=env, timeout=timeout,
                       cwd=ROOT)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    return [json.loads(line) for line in r.stdout.splitlines() if line.startswith("{")]


def test_reference_arm_line_contract():
    lines = _run(["--impl", "reference", "--steps", "1", "--warmup", "0"])
    assert len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["unit"] == "voxels/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["config"]["voxels"] > 4_000_000
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "voxels/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_do_no_work():
    assert _run(["--impl", "reference", "--gpus", "2"], {"RANK": "1", "WORLD_SIZE": "2"}, timeout=60) == []


def test_single_gpu_ops_answer_unavailable_for_the_reference_arm():
    for op in ("convnext", "c2s", "decode", "mesh"):
        lines = _run(["--impl", "reference", "--op", op], timeout=60)
        assert len(lines) == 1 and lines[0]["impl"] == "reference" and "unavailable" in lines[0]
