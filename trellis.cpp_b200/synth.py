"""Seeded synthetic inputs for the five benchmark configurations (host side, numpy).

Thin wrapper over libtb_synth.so (csrc/tb_synth.c). Every voxel decision is a pure
function of (coordinate, seed), so the sets are identical on every host and thread count.
Coordinates are int32 [N,4] = (b=0, x, y, z) in x-major lexicographic order.

  C1  grid 64,   Euclidean band 22 <= |p-c| < 24, each voxel kept with p=0.95 (seed 1)
  C2  grid 256,  shell |d - (100 + 8 n(p))| < 1, noise spacings 32/16/8 (seed 2)
  C3  the C2 shell; children kept where |d - r| < 0.5 at the child centre (seed 2)
  C4  grid 1024, shell |d - (440 + 16 n(p))| < 1, noise spacings 128/64/32 (seed 4)
  C4s grid 512,  half-scale C4 (r=220+-8, spacings 64/32/16) for profiler captures
  C5  grid 512,  4096 boxes, edges U{4..32} per axis, union kept with p=0.3 (seed 5)
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

_lib = None
_i32pp = ctypes.POINTER(ctypes.POINTER(ctypes.c_int32))


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_build.SYNTH_LIB):
            raise FileNotFoundError(f"{_build.SYNTH_LIB} missing; run trellis.cpp_b200/build.py")
        L = ctypes.CDLL(_build.SYNTH_LIB)
        L.tbs_shell.restype = ctypes.c_int64
        L.tbs_shell.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                ctypes.c_uint64, ctypes.c_double, ctypes.c_int, _i32pp]
        L.tbs_band.restype = ctypes.c_int64
        L.tbs_band.argtypes = [ctypes.c_int, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                               ctypes.c_uint64, ctypes.c_int, _i32pp]
        L.tbs_boxes.restype = ctypes.c_int64
        L.tbs_boxes.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_double,
                                ctypes.c_uint64, ctypes.c_int, _i32pp]
        L.tbs_child_mask.restype = None
        L.tbs_child_mask.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_int64, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                     ctypes.c_uint64, ctypes.c_double, ctypes.POINTER(ctypes.c_uint8)]
        L.tbs_noise.restype = ctypes.c_double
        L.tbs_noise.argtypes = [ctypes.c_double] * 4 + [ctypes.c_uint64]
        L.tbs_free.restype = None
        L.tbs_free.argtypes = [ctypes.c_void_p]
        _lib = L
    return _lib


def _take(n, ptr) -> np.ndarray:
    if n < 0:
        raise MemoryError("synthetic generator failed")
    try:
        a = np.ctypeslib.as_array(ptr, shape=(max(n, 1) * 3,))[: n * 3].reshape(n, 3).copy()
    finally:
        _load().tbs_free(ptr)
    out = np.zeros((n, 4), dtype=np.int32)
    out[:, 1:] = a
    return out


def _threads(nthreads):
    return nthreads or min(os.cpu_count() or 1, 64)


def shell(res, radius, amp, spacing0, seed, thick=2.0, nthreads=None) -> np.ndarray:
    p = ctypes.POINTER(ctypes.c_int32)()
    n = _load().tbs_shell(res, radius, amp, spacing0, seed, thick, _threads(nthreads), ctypes.byref(p))
    return _take(n, p)


def band(res, rmin, rmax, keep_p, seed, nthreads=None) -> np.ndarray:
    p = ctypes.POINTER(ctypes.c_int32)()
    n = _load().tbs_band(res, rmin, rmax, keep_p, seed, _threads(nthreads), ctypes.byref(p))
    return _take(n, p)


def boxes(res, nbox, emin, emax, keep_p, seed, nthreads=None) -> np.ndarray:
    p = ctypes.POINTER(ctypes.c_int32)()
    n = _load().tbs_boxes(res, nbox, emin, emax, keep_p, seed, _threads(nthreads), ctypes.byref(p))
    return _take(n, p)


def child_mask(coords, res, radius, amp, spacing0, seed, half=0.5) -> np.ndarray:
    c = np.ascontiguousarray(coords, dtype=np.int32)
    n, stride = c.shape
    m = np.empty((n, 8), dtype=np.uint8)
    _load().tbs_child_mask(c.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n, stride, res, radius, amp,
                           spacing0, seed, half, m.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    return m


# ---- the benchmark configurations -------------------------------------------------------
CONFIGS = {
    "c1": dict(desc="grid 64 band 22<=|p-c|<24 keep 0.95, C=64 fp32", ci=64, co=64, dtype="f32"),
    "c2": dict(desc="grid 256 noisy shell r=100+-8, C=256 f16", ci=256, co=256, dtype="f16"),
    "c3": dict(desc="C2 shell subdivided, ~1M children kept, C=128 bf16", ci=128, co=128, dtype="bf16"),
    "c4": dict(desc="grid 1024 noisy shell r=440+-16, two convs C=64 bf16", ci=64, co=64, dtype="bf16"),
    "c5_32": dict(desc="grid 512, 4096 boxes density 0.3, C=32 f16", ci=32, co=32, dtype="f16"),
    "c5_512": dict(desc="grid 512, 4096 boxes density 0.3, C=512 f16", ci=512, co=512, dtype="f16"),
}


def coords_for(name: str, nthreads=None) -> np.ndarray:
    """Voxel coordinates (int32 [N,4]) of a configuration (C3: the parent shell)."""
    if name == "c1":
        return band(64, 22.0, 24.0, 0.95, 1, nthreads)
    if name in ("c2", "c3"):
        return shell(256, 100.0, 8.0, 32.0, 2, 2.0, nthreads)
    if name == "c4":
        return shell(1024, 440.0, 16.0, 128.0, 4, 2.0, nthreads)
    if name == "c4s":   # half-scale C4 for profiler captures (still larger than L2)
        return shell(512, 220.0, 8.0, 64.0, 4, 2.0, nthreads)
    if name.startswith("c5"):
        return boxes(512, 4096, 4, 32, 0.3, 5, nthreads)
    raise KeyError(name)


def c3_mask(parents: np.ndarray) -> np.ndarray:
    """Seeded thickness mask [N,8] of configuration C3 (the external-mask path of sparse_c2s)."""
    return child_mask(parents, 256, 100.0, 8.0, 32.0, 2, 0.5)
