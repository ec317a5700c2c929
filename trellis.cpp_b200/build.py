"""Build the sparse-conv library in-tree: trellis.cpp_b200/libtb_sparse.so (sm_100a).

nvcc compiles every csrc/*.cu for `-gencode arch=compute_100a,code=sm_100a` and the C++
host mirror (csrc/*.cpp); the result links cudart statically, so the .so carries no
dependence on a particular libcudart next to torch's. Objects go to _build/ (git-ignored).
Run `python trellis.cpp_b200/build.py [-v]`; -v prints ptxas register/smem usage.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libtb_sparse.so")
SYNTH_LIB = os.path.join(PKG, "libtb_synth.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("command failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stdout + r.stderr


def build(verbose: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu"))) + sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    synth_src = os.path.join(CSRC, "tb_synth.c")
    if force or not os.path.exists(SYNTH_LIB) or os.path.getmtime(SYNTH_LIB) < os.path.getmtime(synth_src):
        # host-only generator library; strict FP so every host computes the same voxel sets
        _run(["gcc", "-O2", "-ffp-contract=off", "-fPIC", "-shared", "-pthread", "-std=c11",
              "-o", SYNTH_LIB, synth_src, "-lm"])
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")) \
        + glob.glob(os.path.join(INCLUDE, "*.hpp"))
    newest_header = max(os.path.getmtime(h) for h in headers)
    common = ["-O3", "-std=c++17", "-I", INCLUDE, "-I", CSRC, "-Xcompiler", "-fPIC,-Wall"]
    jobs = []
    objs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if not force and os.path.exists(obj) and os.path.getmtime(obj) > max(os.path.getmtime(src), newest_header):
            continue
        if src.endswith(".cu"):
            cmd = [NVCC, *ARCH, "-lineinfo", *common, "-c", src, "-o", obj]
            if verbose:
                cmd += ["-Xptxas", "-v"]
        else:
            cmd = [NVCC, *common, "-x", "c++", "-c", src, "-o", obj]
        jobs.append(cmd)
    with ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for out in ex.map(_run, jobs):
            if verbose and out.strip():
                print(out)
    if force or jobs or not os.path.exists(LIB):
        _run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lrt"])
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
