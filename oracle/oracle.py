"""CPU oracle for the sparse submanifold-conv path -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes front end over ``tb_oracle.c`` (the C restatement of the reference's
``src/sparse.cpp``). Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and its ``--impl reference`` arm) import this module; the product
library never does.

Functions and the reference lines they follow (paths inside pwilkin/trellis.cpp):

* :func:`build_neighbor_table` -- ``src/sparse.cpp:21-39``
* :func:`submconv` -- ``src/sparse.cpp:64-92`` (fp64 accumulation of the given operands)
* :func:`submconv_rows` -- the same for a subset of output rows
* :func:`submconv_f32_mt` -- the same loop in fp32 on host threads (timed CPU baseline)
* :func:`subdivide` -- ``src/sparse.cpp:205-222``
* :func:`c2s_gather` -- ``src/sparse.cpp:263-266,288``
* :func:`c2s_block` -- the whole ``sparse_c2s`` data flow, ``src/sparse.cpp:172-336``
  (LayerNorm/SiLU in numpy, convs through the C restatement)
* :func:`dual_grid_mesh` -- ``src/dual_grid.cpp:16-56``
* :func:`ref_dual_grid_mesh` -- the reference's own ``dual_grid_to_mesh``, compiled from its
  sources into ``oracle/_ref/`` (only where those sources were present at build time)
* :func:`ref_build_neighbor_table` -- the reference's own ``build_neighbor_table``
  (``src/sparse.cpp:21-39``, its ``std::unordered_map`` loop), compiled likewise
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "liboracle.so")
REF_MESH_SO = os.path.join(_HERE, "_ref", "libref_dual_grid.so")
REF_NBR_SO = os.path.join(_HERE, "_ref", "libref_nbr.so")
_lib = None
_ref_mesh = None
_ref_nbr = None

_i32p = ctypes.POINTER(ctypes.c_int32)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)


def build() -> str:
    """Compile ``liboracle.so`` with the committed Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(
                os.path.join(_HERE, "tb_oracle.c")):
            build()
        L = ctypes.CDLL(_SO)
        L.orc_key.restype = ctypes.c_uint64
        L.orc_key.argtypes = [ctypes.c_int32] * 4
        L.orc_build_neighbor_table.restype = ctypes.c_int
        L.orc_build_neighbor_table.argtypes = [_i32p, ctypes.c_int64, ctypes.c_int, _i32p]
        L.orc_submconv_f64.restype = ctypes.c_int
        L.orc_submconv_f64.argtypes = [_i32p, ctypes.c_int64, _f32p, ctypes.c_int, _f32p,
                                       _f32p, ctypes.c_int, ctypes.c_int, _f64p]
        L.orc_submconv_rows_f64.restype = ctypes.c_int
        L.orc_submconv_rows_f64.argtypes = [_i32p, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64), ctypes.c_int64,
                                            _f32p, ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int,
                                            _f64p]
        L.orc_weight_tap_major.restype = None
        L.orc_weight_tap_major.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, _f32p]
        L.orc_submconv_f32_mt.restype = ctypes.c_int
        L.orc_submconv_f32_mt.argtypes = [_i32p, ctypes.c_int64, _f32p, ctypes.c_int, _f32p,
                                          _f32p, ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int]
        L.orc_submconv_f32_mt_range.restype = ctypes.c_int
        L.orc_submconv_f32_mt_range.argtypes = [_i32p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, _f32p,
                                                ctypes.c_int, _f32p, _f32p, ctypes.c_int, ctypes.c_int, _f32p,
                                                ctypes.c_int]
        L.orc_subdivide.restype = ctypes.c_int64
        L.orc_subdivide.argtypes = [_i32p, ctypes.c_int64, ctypes.c_int, _u8p, _i32p, _i32p, _i32p]
        L.orc_c2s_gather.restype = None
        L.orc_c2s_gather.argtypes = [_f32p, _i32p, ctypes.c_int64, ctypes.c_int, _f32p]
        L.orc_count_valid.restype = ctypes.c_int64
        L.orc_count_valid.argtypes = [_i32p, ctypes.c_int64]
        L.orc_dual_grid_mesh.restype = ctypes.c_int64
        L.orc_dual_grid_mesh.argtypes = [_i32p, ctypes.c_int64, _f32p, ctypes.c_int, _f32p, _i32p, _f32p]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def key(b: int, x: int, y: int, z: int) -> int:
    """The packed coordinate key (``src/sparse.cpp:25``; batch folded into bits 60..63)."""
    return int(lib().orc_key(b, x, y, z))


def build_neighbor_table(coords: np.ndarray) -> np.ndarray:
    """Tap-major int32 ``[27*N]`` neighbor map, sentinel N (``src/sparse.cpp:21-39``).

    ``coords`` is int32 ``[N,3]`` (x,y,z) or ``[N,4]`` (b,x,y,z)."""
    c = np.ascontiguousarray(coords, dtype=np.int32)
    n, stride = c.shape
    out = np.empty(27 * n, dtype=np.int32)
    if lib().orc_build_neighbor_table(_p(c, _i32p), n, stride, _p(out, _i32p)) != 0:
        raise ValueError("orc_build_neighbor_table failed")
    return out


def count_valid(nbr: np.ndarray, n: int) -> int:
    a = np.ascontiguousarray(nbr, dtype=np.int32)
    return int(lib().orc_count_valid(_p(a, _i32p), n))


def submconv(nbr: np.ndarray, feats: np.ndarray, weight: np.ndarray, bias=None,
             silu: bool = False) -> np.ndarray:
    """fp64 submanifold conv (``src/sparse.cpp:64-92``).

    feats float32 ``[N,Ci]``, weight float32 ``[Co,27,Ci]`` (or ``[Co,3,3,3,Ci]``), bias
    ``[Co]`` or None. Returns float64 ``[N,Co]``."""
    f = np.ascontiguousarray(feats, dtype=np.float32)
    n, ci = f.shape
    w = np.ascontiguousarray(weight, dtype=np.float32).reshape(weight.shape[0], 27, ci)
    co = w.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    nb = np.ascontiguousarray(nbr, dtype=np.int32)
    out = np.empty((n, co), dtype=np.float64)
    rc = lib().orc_submconv_f64(_p(nb, _i32p), n, _p(f, _f32p), ci, _p(w, _f32p),
                                None if b is None else _p(b, _f32p), co, 1 if silu else 0,
                                _p(out, _f64p))
    if rc != 0:
        raise ValueError("orc_submconv_f64 failed")
    return out


def submconv_rows(nbr, feats, weight, rows, bias=None, silu: bool = False) -> np.ndarray:
    """:func:`submconv` for the output rows ``rows`` only; returns float64 [len(rows), Co]."""
    f = np.ascontiguousarray(feats, dtype=np.float32)
    n, ci = f.shape
    w = np.ascontiguousarray(weight, dtype=np.float32).reshape(weight.shape[0], 27, ci)
    co = w.shape[0]
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    r = np.ascontiguousarray(rows, dtype=np.int64)
    nb = np.ascontiguousarray(nbr, dtype=np.int32)
    out = np.empty((r.size, co), dtype=np.float64)
    rc = lib().orc_submconv_rows_f64(_p(nb, _i32p), n, r.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), r.size,
                                     _p(f, _f32p), ci, _p(w, _f32p), None if b is None else _p(b, _f32p), co,
                                     1 if silu else 0, _p(out, _f64p))
    if rc != 0:
        raise ValueError("orc_submconv_rows_f64 failed")
    return out


def weight_tap_major(weight: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(weight, dtype=np.float32)
    co = w.shape[0]
    ci = w.shape[-1]
    wt = np.empty((27, ci, co), dtype=np.float32)
    lib().orc_weight_tap_major(_p(w, _f32p), ci, co, _p(wt, _f32p))
    return wt


def submconv_f32_mt(nbr, feats, wt, bias=None, silu=False, nthreads=None, out=None):
    """fp32 multi-threaded conv (the timed CPU baseline). ``wt`` from :func:`weight_tap_major`."""
    f = np.ascontiguousarray(feats, dtype=np.float32)
    n, ci = f.shape
    co = wt.shape[2]
    if out is None:
        out = np.empty((n, co), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    nb = np.ascontiguousarray(nbr, dtype=np.int32)
    nt = nthreads or os.cpu_count() or 1
    rc = lib().orc_submconv_f32_mt(_p(nb, _i32p), n, _p(f, _f32p), ci, _p(wt, _f32p),
                                   None if b is None else _p(b, _f32p), co, 1 if silu else 0,
                                   _p(out, _f32p), nt)
    if rc != 0:
        raise ValueError("orc_submconv_f32_mt failed")
    return out


def submconv_f32_mt_range(nbr, feats, wt, row0, nrows, bias=None, silu=False, nthreads=None, out=None):
    """Rows [row0, row0+nrows) of :func:`submconv_f32_mt` (a bounded sample for timing)."""
    f = np.ascontiguousarray(feats, dtype=np.float32)
    n, ci = f.shape
    co = wt.shape[2]
    if out is None:
        out = np.empty((n, co), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    nb = np.ascontiguousarray(nbr, dtype=np.int32)
    nt = nthreads or os.cpu_count() or 1
    rc = lib().orc_submconv_f32_mt_range(_p(nb, _i32p), n, row0, nrows, _p(f, _f32p), ci, _p(wt, _f32p),
                                         None if b is None else _p(b, _f32p), co, 1 if silu else 0,
                                         _p(out, _f32p), nt)
    if rc != 0:
        raise ValueError("orc_submconv_f32_mt_range failed")
    return out


def subdivide(coords: np.ndarray, mask: np.ndarray):
    """Octant subdivide (``src/sparse.cpp:205-222``): returns (child coords, gidx, mstart)."""
    c = np.ascontiguousarray(coords, dtype=np.int32)
    n, stride = c.shape
    m8 = np.ascontiguousarray(mask, dtype=np.uint8).reshape(-1)
    assert m8.size == 8 * n
    mtot = int(m8.astype(bool).sum())
    child = np.empty((mtot, stride), dtype=np.int32)
    gidx = np.empty(mtot, dtype=np.int32)
    mstart = np.empty(n + 1, dtype=np.int32)
    m = lib().orc_subdivide(_p(c, _i32p), n, stride, _p(m8, _u8p), _p(child, _i32p),
                            _p(gidx, _i32p), _p(mstart, _i32p))
    assert m == mtot
    return child, gidx, mstart


def c2s_gather(src: np.ndarray, gidx: np.ndarray, c: int) -> np.ndarray:
    """Child m takes row gidx[m] of the ``[8N, C]`` view of conv1's output."""
    s = np.ascontiguousarray(src, dtype=np.float32).reshape(-1)
    g = np.ascontiguousarray(gidx, dtype=np.int32)
    out = np.empty((g.size, c), dtype=np.float32)
    lib().orc_c2s_gather(_p(s, _f32p), _p(g, _i32p), g.size, c, _p(out, _f32p))
    return out


def layer_norm(x: np.ndarray, w=None, b=None, eps: float = 1e-6) -> np.ndarray:
    """Row LayerNorm over channels, as ggml_norm + affine (``src/sparse.cpp:259-260,293``)."""
    x = x.astype(np.float64)
    mu = x.mean(axis=1, keepdims=True)
    var = ((x - mu) ** 2).mean(axis=1, keepdims=True)
    y = (x - mu) / np.sqrt(var + eps)
    if w is not None:
        y = y * w.astype(np.float64)
    if b is not None:
        y = y + b.astype(np.float64)
    return y


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


def c2s_block(coords, feats, w, cout, ext_mask=None):
    """The ``sparse_c2s`` data flow (``src/sparse.cpp:172-336``) on the CPU.

    ``w`` holds float32 arrays: ``to_subdiv.weight [8,Cin]``, ``to_subdiv.bias [8]``,
    ``norm1.weight/bias [Cin]``, ``conv1.weight [8*Cout,27,Cin]``, ``conv1.bias``,
    ``conv2.weight [Cout,27,Cout]``, ``conv2.bias``. Returns (out [M,Cout], child coords,
    mask [N,8])."""
    feats = np.asarray(feats, dtype=np.float32)
    n, cin = feats.shape
    if ext_mask is None:
        logits = feats.astype(np.float64) @ w["to_subdiv.weight"].astype(np.float64).T \
            + w["to_subdiv.bias"].astype(np.float64)                       # :184-190
        mask = (logits > 0).astype(np.uint8)                                 # :215
    else:
        mask = np.asarray(ext_mask, dtype=np.uint8).reshape(n, 8)
    nbr = build_neighbor_table(coords)                                       # :177
    h = silu(layer_norm(feats, w["norm1.weight"], w["norm1.bias"]))          # :259-261
    h1 = submconv(nbr, h.astype(np.float32), w["conv1.weight"], w["conv1.bias"])  # :286
    child, gidx, _ = subdivide(coords, mask)                                 # :205-222
    hc = c2s_gather(h1.astype(np.float32), gidx, cout)                       # :288
    hn = silu(layer_norm(hc))                                                # :293
    nbr2 = build_neighbor_table(child)                                       # :224
    o = submconv(nbr2, hn.astype(np.float32), w["conv2.weight"], w["conv2.bias"])  # :319
    k = cin // 8
    xs = c2s_gather(feats, gidx, k)                                          # :307
    o = o + np.repeat(xs.astype(np.float64), cout // k, axis=1)              # :322-323
    return o, child, mask


def dual_grid_mesh(coords: np.ndarray, feats7: np.ndarray, res: int):
    """``dual_grid_to_mesh`` (``src/dual_grid.cpp:16-56``): returns (verts [N,3] f32, faces
    [F,3] int32, gap [F/2] f32), gap = the relative margin of each quad's split decision."""
    c = np.ascontiguousarray(coords, dtype=np.int32)
    f7 = np.ascontiguousarray(feats7, dtype=np.float32)
    n = c.shape[0]
    assert c.shape == (n, 3) and f7.shape == (n, 7)
    verts = np.empty((n, 3), dtype=np.float32)
    faces = np.empty((6 * n, 3), dtype=np.int32)
    gap = np.empty(3 * n, dtype=np.float32)
    f = lib().orc_dual_grid_mesh(_p(c, _i32p), n, _p(f7, _f32p), res, _p(verts, _f32p), _p(faces, _i32p),
                                 _p(gap, _f32p))
    if f < 0:
        raise MemoryError("orc_dual_grid_mesh: allocation failed")
    return verts, faces[:f].copy(), gap[:f // 2].copy()


def ref_available() -> bool:
    return os.path.exists(REF_MESH_SO)


def ref_dual_grid_mesh(coords: np.ndarray, feats7: np.ndarray, res: int):
    """The reference's own ``trellis::dual_grid_to_mesh`` (``oracle/_ref``): (verts, faces)."""
    global _ref_mesh
    if _ref_mesh is None:
        L = ctypes.CDLL(REF_MESH_SO)
        L.ref_dual_grid_mesh.restype = ctypes.c_int64
        L.ref_dual_grid_mesh.argtypes = [_i32p, ctypes.c_int64, _f32p, ctypes.c_int, _f32p, _i32p, ctypes.c_int64]
        _ref_mesh = L
    c = np.ascontiguousarray(coords, dtype=np.int32)
    f7 = np.ascontiguousarray(feats7, dtype=np.float32)
    n = c.shape[0]
    verts = np.empty((n, 3), dtype=np.float32)
    faces = np.empty((6 * n, 3), dtype=np.int32)
    f = _ref_mesh.ref_dual_grid_mesh(_p(c, _i32p), n, _p(f7, _f32p), res, _p(verts, _f32p), _p(faces, _i32p),
                                     6 * n)
    return verts, faces[:f].copy()


def ref_nbr_available() -> bool:
    return os.path.exists(REF_NBR_SO)


def ref_build_neighbor_table(coords: np.ndarray) -> np.ndarray:
    """The reference's own ``trellis::build_neighbor_table`` (``oracle/_ref``), single-threaded:
    tap-major int32 ``[27*N]``, sentinel N. Coordinates int32 [N,3] or [N,4] (batch ignored, as
    the reference's (x,y,z) table has no batch)."""
    global _ref_nbr
    if _ref_nbr is None:
        L = ctypes.CDLL(REF_NBR_SO)
        L.ref_build_neighbor_table.restype = ctypes.c_int
        L.ref_build_neighbor_table.argtypes = [_i32p, ctypes.c_int64, ctypes.c_int, _i32p]
        _ref_nbr = L
    c = np.ascontiguousarray(coords, dtype=np.int32)
    n, stride = c.shape
    out = np.empty(27 * n, dtype=np.int32)
    if _ref_nbr.ref_build_neighbor_table(_p(c, _i32p), n, stride, _p(out, _i32p)) != 0:
        raise ValueError("ref_build_neighbor_table failed")
    return out
