"""Host-side operator mirror of the reference's sparse op layer, over the C ABI.

Names and argument meanings follow pwilkin/trellis.cpp's ``include/sparse.h``:

* :func:`build_neighbor_table` -- ``trellis::build_neighbor_table`` (sparse.h:14-17)
* :func:`sparse_submconv` -- ``trellis::sparse_submconv`` (sparse.h:19-22), with explicit
  weight / bias tensors in place of a Model + name prefix
* :func:`subdivide` / :func:`c2s_gather` -- the subdivide and channel-to-spatial steps of
  ``trellis::sparse_c2s`` (src/sparse.cpp:205-222, 263-266, 288, 307)
* :func:`sparse_convnext` / :func:`convnext_tail` -- ``trellis::sparse_convnext``
  (sparse.h:23-25) and its LayerNorm / MLP / residual tail
* :func:`sparse_c2s` -- ``trellis::sparse_c2s`` (sparse.h:27-35), the whole C2S up-block
* :func:`submconv_stack_host` -- a host-buffer stage run (upload, map, convs, read back), the
  shape of ``run1`` / ``GraphRun::run`` (src/shape_decoder.cpp:34-51)

Device tensors are torch CUDA tensors used only as memory; every computation runs in
libtb_sparse.so. Errors raise :class:`TBError` (the reference throws std::runtime_error).
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib
from ._lib import TBError, check  # noqa: F401

_DT = {torch.float32: _lib.TB_F32, torch.float16: _lib.TB_F16, torch.bfloat16: _lib.TB_BF16}
_EPI = {"none": _lib.TB_EPI_NONE, None: _lib.TB_EPI_NONE, "silu": _lib.TB_EPI_SILU}
_ctxs: dict = {}

# Kernels one tb_build_neighbor_map call launches: the order and range check, then five that
# branch on the layout decided on the device (sorted, block or voxel hash); with the sorted
# layout the last two return at once.
NBR_MAP_LAUNCHES = 6


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def context(device=None):
    """The per-device tb_ctx, bound to torch's current stream on that device (the current device
    when `device` is None or names no index). One context per device is shared by every caller
    in the process; like the C contexts it wraps, it is not safe to use from two threads at once."""
    idx = None if device is None else torch.device(device).index
    dev = torch.device("cuda", torch.cuda.current_device() if idx is None else idx)
    lib = _lib.load()
    h = _ctxs.get(dev.index)
    stream = torch.cuda.current_stream(dev).cuda_stream
    if h is None:
        h = ctypes.c_void_p()
        check(lib.tb_ctx_create(dev.index, ctypes.c_void_p(stream), ctypes.byref(h)), "tb_ctx_create")
        _ctxs[dev.index] = h
    else:
        check(lib.tb_ctx_set_stream(h, ctypes.c_void_p(stream)), "tb_ctx_set_stream", h)
    return h


def set_conv_path(path: str = "auto", device=None):
    """Select the tensor-core conv kernel: "auto", "gather", "brick" or "pair" (tuning/testing)."""
    ctx = context(device)
    code = {"auto": _lib.TB_CONV_AUTO, "gather": _lib.TB_CONV_GATHER, "brick": _lib.TB_CONV_BRICK,
            "pair": _lib.TB_CONV_PAIR}[path]
    check(_lib.load().tb_ctx_set_conv_path(ctx, code), "tb_ctx_set_conv_path", ctx)


def check_device(device=None):
    """Synchronise and raise if a kernel reported a failed device-side check."""
    ctx = context(device)
    check(_lib.load().tb_ctx_check_device(ctx), "tb_ctx_check_device", ctx)


def _need_cuda(*ts):
    for t in ts:
        if t is not None and (not t.is_cuda or not t.is_contiguous()):
            raise ValueError("expected contiguous CUDA tensors")


def build_neighbor_table(coords: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Tap-major int32 [27*N] neighbor map (sentinel N) of int32 coords [N,3] or [N,4]."""
    _need_cuda(coords)
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] not in (3, 4):
        raise ValueError("coords must be int32 [N,3] or [N,4]")
    n = coords.shape[0]
    if out is None:
        out = torch.empty(27 * n, dtype=torch.int32, device=coords.device)
    ctx = context(coords.device)
    check(_lib.load().tb_build_neighbor_map(ctx, _ptr(coords), n, coords.shape[1], _ptr(out)),
          "tb_build_neighbor_map", ctx)
    return out


def count_valid_pairs(nbr: torch.Tensor, n: int) -> int:
    _need_cuda(nbr)
    ctx = context(nbr.device)
    v = ctypes.c_int64()
    check(_lib.load().tb_count_valid_pairs(ctx, _ptr(nbr), n, ctypes.byref(v)), "tb_count_valid_pairs", ctx)
    return int(v.value)


def sparse_submconv(feats: torch.Tensor, nbr: torch.Tensor, weight: torch.Tensor,
                    bias: torch.Tensor | None = None, epi: str = "none", out_dtype=None,
                    out: torch.Tensor | None = None) -> torch.Tensor:
    """out = epi(bias + sum_t W_t . feats[nbr_t]), feats [N,Ci], weight [Co,27,Ci] or
    [Co,3,3,3,Ci] (same dtype as feats), bias float32 [Co] or None."""
    _need_cuda(feats, nbr, weight, bias)
    if feats.dtype not in _DT or weight.dtype != feats.dtype:
        raise ValueError("feats and weight must share a dtype among float32/float16/bfloat16")
    n, ci = feats.shape
    co = weight.shape[0]
    if weight.numel() != co * 27 * ci:
        raise ValueError("weight must be [Co,27,Ci]")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != co):
        raise ValueError("bias must be float32 [Co]")
    if nbr.numel() != 27 * n:
        raise ValueError("nbr must have 27*N entries")
    od = feats.dtype if out_dtype is None else out_dtype
    if out is None:
        out = torch.empty((n, co), dtype=od, device=feats.device)
    ctx = context(feats.device)
    check(_lib.load().tb_submconv(ctx, _ptr(nbr), n, _ptr(feats), ci, _ptr(weight), _ptr(bias), co,
                                  _DT[feats.dtype], _DT[od], _EPI[epi], _ptr(out)), "tb_submconv", ctx)
    return out


def sparse_submconv_range(feats: torch.Tensor, nbr: torch.Tensor, weight: torch.Tensor, bias, row0: int, nrows: int,
                          out: torch.Tensor, epi: str = "none") -> torch.Tensor:
    """Rows [row0, row0 + nrows) of :func:`sparse_submconv` written into ``out`` [N,Co] (the
    reference's ``submconv_range``, src/sparse.cpp:64-79); any row0."""
    _need_cuda(feats, nbr, weight, bias, out)
    n, ci = feats.shape
    co = weight.shape[0]
    if weight.dtype != feats.dtype or weight.numel() != co * 27 * ci or nbr.numel() != 27 * n:
        raise ValueError("weight must be [Co,27,Ci] of feats' dtype and nbr 27*N")
    if out.shape != (n, co):
        raise ValueError("out must be [N, Co]")
    ctx = context(feats.device)
    check(_lib.load().tb_submconv_range(ctx, _ptr(nbr), n, row0, nrows, _ptr(feats), ci, _ptr(weight), _ptr(bias), co,
                                        _DT[feats.dtype], _DT[out.dtype], _EPI[epi], _ptr(out)),
          "tb_submconv_range", ctx)
    return out


def _f32_vec(t, n, name):
    if t is None or not t.is_cuda or t.dtype != torch.float32 or t.numel() != n or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous float32 CUDA tensor of {n} values")


def convnext_tail(h: torch.Tensor, x: torch.Tensor, norm_w, norm_b, w1, b1, w2, b2, out_dtype=None,
                  out: torch.Tensor | None = None) -> torch.Tensor:
    """The per-voxel tail of ``sparse_convnext`` (src/sparse.cpp:124-133):
    ``x + W2 . silu(W1 . LN(h) + b1) + b2`` with LN over channels (eps 1e-6, affine).

    h [N,C] float32 or x's dtype; x [N,C]; w1 [4C,C] and w2 [C,4C] in x's dtype; norm_w, norm_b,
    b1, b2 float32."""
    _need_cuda(h, x, w1, w2)
    if x.dtype not in _DT or w1.dtype != x.dtype or w2.dtype != x.dtype:
        raise ValueError("x, w1 and w2 must share a dtype among float32/float16/bfloat16")
    if h.dtype not in (torch.float32, x.dtype) or h.shape != x.shape:
        raise ValueError("h must be [N,C] float32 or x's dtype")
    n, c = x.shape
    if w1.numel() != 4 * c * c or w2.numel() != 4 * c * c:
        raise ValueError("w1 must be [4C,C] and w2 [C,4C]")
    for t, m, name in ((norm_w, c, "norm_w"), (norm_b, c, "norm_b"), (b1, 4 * c, "b1"), (b2, c, "b2")):
        _f32_vec(t, m, name)
    od = x.dtype if out_dtype is None else out_dtype
    if out is None:
        out = torch.empty((n, c), dtype=od, device=x.device)
    ctx = context(x.device)
    check(_lib.load().tb_convnext_tail(ctx, n, c, _ptr(h), _DT[h.dtype], _ptr(x), _ptr(norm_w), _ptr(norm_b),
                                       _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2), _DT[x.dtype], _DT[od], _ptr(out)),
          "tb_convnext_tail", ctx)
    return out


def sparse_convnext(feats: torch.Tensor, nbr: torch.Tensor, conv_w, conv_b, norm_w, norm_b, w1, b1, w2, b2,
                    out_dtype=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """``trellis::sparse_convnext`` (include/sparse.h:23-25): conv (weight [C,27,C], bias [C]),
    then :func:`convnext_tail` with the block input ``feats`` as the residual."""
    _need_cuda(feats, nbr, conv_w, w1, w2)
    n, c = feats.shape
    if conv_w.dtype != feats.dtype or w1.dtype != feats.dtype or w2.dtype != feats.dtype:
        raise ValueError("weights must share feats' dtype")
    if conv_w.numel() != c * 27 * c or nbr.numel() != 27 * n:
        raise ValueError("conv weight must be [C,27,C] and nbr 27*N")
    if conv_b is not None:
        _f32_vec(conv_b, c, "conv_b")
    for t, m, name in ((norm_w, c, "norm_w"), (norm_b, c, "norm_b"), (b1, 4 * c, "b1"), (b2, c, "b2")):
        _f32_vec(t, m, name)
    od = feats.dtype if out_dtype is None else out_dtype
    if out is None:
        out = torch.empty((n, c), dtype=od, device=feats.device)
    ctx = context(feats.device)
    check(_lib.load().tb_sparse_convnext(ctx, _ptr(nbr), n, _ptr(feats), c, _ptr(conv_w), _ptr(conv_b),
                                         _ptr(norm_w), _ptr(norm_b), _ptr(w1), _ptr(b1), _ptr(w2), _ptr(b2),
                                         _DT[feats.dtype], _DT[od], _ptr(out)), "tb_sparse_convnext", ctx)
    return out


def subdivide(coords: torch.Tensor, mask: torch.Tensor, max_children: int | None = None):
    """(child coords [M,s], gidx [M], mstart [N+1]) for uint8/bool mask [N,8]."""
    _need_cuda(coords, mask)
    n, s = coords.shape
    m8 = mask.to(torch.uint8).contiguous() if mask.dtype != torch.uint8 else mask
    if max_children is None:
        max_children = 8 * n
    child = torch.empty((max_children, s), dtype=torch.int32, device=coords.device)
    gidx = torch.empty(max_children, dtype=torch.int32, device=coords.device)
    mstart = torch.empty(n + 1, dtype=torch.int32, device=coords.device)
    m = ctypes.c_int64()
    ctx = context(coords.device)
    check(_lib.load().tb_subdivide(ctx, _ptr(coords), n, s, _ptr(m8), _ptr(child), _ptr(gidx), _ptr(mstart),
                                   max_children, ctypes.byref(m)), "tb_subdivide", ctx)
    return child[: m.value], gidx[: m.value], mstart


def dual_grid_mesh(coords: torch.Tensor, feats7: torch.Tensor, res: int, max_faces: int | None = None):
    """trellis::dual_grid_to_mesh (src/dual_grid.cpp:16-56) on the device: (verts [N,3] float32,
    faces [F,3] int32) from int32 coords [N,3|4] and the decoder head's float32 [N,7] fields."""
    _need_cuda(coords, feats7)
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] not in (3, 4):
        raise ValueError("coords must be int32 [N,3] or [N,4]")
    n, s = coords.shape
    if feats7.dtype != torch.float32 or tuple(feats7.shape) != (n, 7):
        raise ValueError("feats7 must be a contiguous float32 [N, 7] tensor")
    if max_faces is None:
        max_faces = 6 * n
    verts = torch.empty((n, 3), dtype=torch.float32, device=coords.device)
    faces = torch.empty((max(max_faces, 1), 3), dtype=torch.int32, device=coords.device)
    f = ctypes.c_int64()
    ctx = context(coords.device)
    check(_lib.load().tb_dual_grid_mesh(ctx, _ptr(coords), n, s, _ptr(feats7), int(res), _ptr(verts), _ptr(faces),
                                        max_faces, ctypes.byref(f)), "tb_dual_grid_mesh", ctx)
    return verts, faces[: f.value]


def linear(a: torch.Tensor, w: torch.Tensor, bias=None, act: str = "none", residual=None, out_dtype=None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """out = act(a @ w.T + bias) + residual (a [M,K], w [N,K] of a's dtype; bias float32 [N])."""
    _need_cuda(a, w, bias, residual)
    m, k = a.shape
    n = w.shape[0]
    if w.dtype != a.dtype or w.shape[1] != k:
        raise ValueError("w must be [N, K] of a's dtype")
    if bias is not None:
        _f32_vec(bias, n, "bias")
    od = a.dtype if out_dtype is None else out_dtype
    if out is None:
        out = torch.empty((m, n), dtype=od, device=a.device)
    rd = residual.dtype if residual is not None else a.dtype
    ctx = context(a.device)
    check(_lib.load().tb_linear(ctx, m, k, n, _ptr(a), _ptr(w), _ptr(bias), _ptr(residual), _DT[rd], _EPI[act],
                                _DT[a.dtype], _DT[out.dtype], _ptr(out)), "tb_linear", ctx)
    return out


def layer_norm(x: torch.Tensor, w=None, b=None, eps: float = 1e-6, act: str = "none", out_dtype=None) -> torch.Tensor:
    """act(LayerNorm(x) * w + b) over the last dim (w, b float32 or None)."""
    _need_cuda(x, w, b)
    n, c = x.shape
    od = x.dtype if out_dtype is None else out_dtype
    out = torch.empty((n, c), dtype=od, device=x.device)
    ctx = context(x.device)
    check(_lib.load().tb_layer_norm(ctx, _ptr(x), _DT[x.dtype], n, c, _ptr(w), _ptr(b), eps, _EPI[act], _DT[od],
                                    _ptr(out)), "tb_layer_norm", ctx)
    return out


def sparse_c2s(coords: torch.Tensor, feats: torch.Tensor, params: dict, cout: int, ext_mask=None,
               out_dtype=None, max_children: int | None = None):
    """``trellis::sparse_c2s`` (include/sparse.h:27-35, src/sparse.cpp:172-336) on the device.

    ``params`` maps the reference's tensor names under the block prefix to CUDA tensors:
    ``to_subdiv.weight`` [8,Cin] / ``to_subdiv.bias`` [8] (float32; unused with ``ext_mask``),
    ``norm1.weight`` / ``norm1.bias`` [Cin] (float32), ``conv1.weight`` [8*Cout,27,Cin] and
    ``conv2.weight`` [Cout,27,Cout] (feats' dtype), ``conv1.bias`` / ``conv2.bias`` (float32 or
    absent). Returns ``(out [M,Cout], child coords [M,s], mask [N,8] uint8)`` -- the fields of
    the reference's ``C2SResult``."""
    _need_cuda(coords, feats)
    n, s = coords.shape
    cin = feats.shape[1]
    dt = feats.dtype
    w1, w2 = params["conv1.weight"], params["conv2.weight"]
    if w1.dtype != dt or w2.dtype != dt:
        raise ValueError("conv weights must share feats' dtype")
    if w1.numel() != 8 * cout * 27 * cin or w2.numel() != cout * 27 * cout:
        raise ValueError("conv1.weight must be [8*Cout,27,Cin] and conv2.weight [Cout,27,Cout]")
    _f32_vec(params["norm1.weight"], cin, "norm1.weight")
    _f32_vec(params["norm1.bias"], cin, "norm1.bias")
    for name, m in (("conv1.bias", 8 * cout), ("conv2.bias", cout)):
        if params.get(name) is not None:
            _f32_vec(params[name], m, name)
    sw, sb = params.get("to_subdiv.weight"), params.get("to_subdiv.bias")
    if ext_mask is None:
        if sw is None or sw.dtype != torch.float32 or sw.numel() != 8 * cin or not sw.is_contiguous():
            raise ValueError("to_subdiv.weight must be a contiguous float32 [8, Cin] tensor")
        if sb is not None:
            _f32_vec(sb, 8, "to_subdiv.bias")
        em = None
    else:
        em = ext_mask.to(torch.uint8).contiguous()
        if em.numel() != 8 * n:
            raise ValueError("ext_mask must have 8*N entries")
    if max_children is None:
        max_children = 8 * n
    od = dt if out_dtype is None else out_dtype
    child = torch.empty((max_children, s), dtype=torch.int32, device=coords.device)
    out = torch.empty((max_children, cout), dtype=od, device=coords.device)
    mask = torch.empty((n, 8), dtype=torch.uint8, device=coords.device)
    prm = _lib.C2SParams(_ptr(sw if em is None else None).value, _ptr(sb if em is None else None).value,
                         _ptr(params["norm1.weight"]).value, _ptr(params["norm1.bias"]).value, _ptr(w1).value,
                         _ptr(params.get("conv1.bias")).value, _ptr(w2).value, _ptr(params.get("conv2.bias")).value)
    m = ctypes.c_int64()
    ctx = context(coords.device)
    check(_lib.load().tb_sparse_c2s(ctx, _ptr(coords.contiguous()), n, s, _ptr(feats), cin, cout, ctypes.byref(prm),
                                    _ptr(em), _DT[dt], _DT[od], max_children, _ptr(child), _ptr(out), _ptr(mask),
                                    ctypes.byref(m)), "tb_sparse_c2s", ctx)
    return out[: m.value], child[: m.value], mask


def c2s_gather(src: torch.Tensor, gidx: torch.Tensor, c: int) -> torch.Tensor:
    """Child m takes row gidx[m] of src viewed as [8N, c]."""
    _need_cuda(src, gidx)
    m = gidx.numel()
    out = torch.empty((m, c), dtype=src.dtype, device=src.device)
    ctx = context(src.device)
    check(_lib.load().tb_c2s_gather(ctx, _ptr(src), _ptr(gidx), m, c, _DT[src.dtype], _ptr(out)),
          "tb_c2s_gather", ctx)
    return out


def bias_act(x: torch.Tensor, bias: torch.Tensor | None = None, epi: str = "silu") -> torch.Tensor:
    _need_cuda(x, bias)
    n, c = x.shape
    ctx = context(x.device)
    check(_lib.load().tb_bias_act(ctx, _ptr(x), n, c, _ptr(bias), _DT[x.dtype], _EPI[epi]), "tb_bias_act", ctx)
    return x


def sort_rows(coords: torch.Tensor) -> torch.Tensor:
    """Stable permutation (int32 [N]) listing the rows of ``coords`` (int32 [N,3] or [N,4]) in
    ascending (b, x, y, z) order (signed, stable), the order the conv kernels read fastest
    (tb_sort_rows)."""
    _need_cuda(coords)
    if coords.dtype != torch.int32 or coords.dim() != 2 or coords.shape[1] not in (3, 4):
        raise ValueError("coords must be int32 [N,3] or [N,4]")
    coords = coords.contiguous()
    n = coords.shape[0]
    perm = torch.empty(max(n, 1), dtype=torch.int32, device=coords.device)[:n]
    ctx = context(coords.device)
    check(_lib.load().tb_sort_rows(ctx, _ptr(coords), n, coords.shape[1], _ptr(perm)), "tb_sort_rows", ctx)
    return perm


def gather_rows(src: torch.Tensor, rows: torch.Tensor) -> torch.Tensor:
    _need_cuda(src, rows)
    m = rows.numel()
    out = torch.empty((m,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    row_bytes = src[0].numel() * src.element_size() if src.shape[0] else 4
    ctx = context(src.device)
    check(_lib.load().tb_gather_rows(ctx, _ptr(src), _ptr(rows), m, row_bytes, _ptr(out)), "tb_gather_rows", ctx)
    return out


def scatter_rows(dst: torch.Tensor, rows: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    """dst[rows[k]] = src[k] (rows int32)."""
    _need_cuda(dst, rows, src)
    m = rows.numel()
    row_bytes = dst[0].numel() * dst.element_size() if dst.shape[0] else 4
    ctx = context(dst.device)
    check(_lib.load().tb_scatter_rows(ctx, _ptr(src), _ptr(rows), m, row_bytes, _ptr(dst)), "tb_scatter_rows", ctx)
    return dst


def zslab_counts(coords: torch.Tensor, z_min: int, nz: int) -> torch.Tensor:
    _need_cuda(coords)
    counts = torch.empty(nz, dtype=torch.int64, device=coords.device)
    ctx = context(coords.device)
    check(_lib.load().tb_zslab_counts(ctx, _ptr(coords), coords.shape[0], coords.shape[1], z_min, nz,
                                      _ptr(counts)), "tb_zslab_counts", ctx)
    return counts


def submconv_stack_host(coords: np.ndarray, feats: np.ndarray, layers, dtype: torch.dtype,
                        out_dtype: torch.dtype, out: np.ndarray | None = None, device=None) -> np.ndarray:
    """Host coords + host feats in, host features out, through ``tb_submconv_stack_host``.

    ``layers`` is a list of (weight, bias, epi) with device weight [Co,27,Ci] / bias [Co].
    ``feats`` holds the raw bits of ``dtype`` (np.uint16 for f16/bf16, float32 for f32)."""
    coords = np.ascontiguousarray(coords, dtype=np.int32)
    n, s = coords.shape
    arr = (_lib.ConvLayer * len(layers))()
    for k, (w, b, epi) in enumerate(layers):
        arr[k].weight = w.data_ptr()
        arr[k].bias = b.data_ptr() if b is not None else None
        arr[k].ci = w.shape[-1]
        arr[k].co = w.shape[0]
        arr[k].epi = _EPI[epi]
    co = layers[-1][0].shape[0]
    if out is None:
        out = np.empty((n, co), dtype=np.float32 if out_dtype == torch.float32 else np.uint16)
    ctx = context(device if device is not None else layers[0][0].device)
    check(_lib.load().tb_submconv_stack_host(
        ctx, coords.ctypes.data_as(ctypes.c_void_p), n, s, feats.ctypes.data_as(ctypes.c_void_p), arr,
        len(layers), _DT[dtype], _DT[out_dtype], out.ctypes.data_as(ctypes.c_void_p)),
        "tb_submconv_stack_host", ctx)
    return out


# ---- model and input files ----------------------------------------------------------------
_GGUF_NP = {0: np.float32, 1: np.float16, 30: np.uint16}   # BF16 read as its raw 16-bit words
GGUF_F32, GGUF_F16, GGUF_BF16 = 0, 1, 30


def _io_check(status: int, call: str):
    if status != _lib.TB_OK:
        d = _lib.load().tb_io_last_error()
        raise TBError(status, call, d.decode() if d else "")


class GgufFile:
    """A GGUF checkpoint (the reference's Model file, src/trellis_model.cpp:96-137), parsed by
    tb_gguf_open. Shapes are given in torch order (ggml's ne reversed): a sparse conv weight
    is [Co, 27, Ci]."""

    def __init__(self, path: str):
        self._g = ctypes.c_void_p()
        _io_check(_lib.load().tb_gguf_open(str(path).encode(), ctypes.byref(self._g)), "tb_gguf_open")
        self.tensors = {}
        lib = _lib.load()
        for i in range(lib.tb_gguf_n_tensors(self._g)):
            name = ctypes.c_char_p()
            typ, nd = _lib._i32(), _lib._i32()
            ne = (_lib._i64 * 4)()
            nb = ctypes.c_uint64()
            _io_check(lib.tb_gguf_tensor_info(self._g, i, ctypes.byref(name), ctypes.byref(typ), ctypes.byref(nd), ne,
                                              ctypes.byref(nb)), "tb_gguf_tensor_info")
            shape = tuple(int(ne[d]) for d in range(nd.value))[::-1]
            try:
                key = name.value.decode("utf-8")
            except UnicodeDecodeError:
                self.close()
                raise TBError(1, "GgufFile", f"tensor {i}: name is not valid UTF-8") from None
            self.tensors[key] = (i, int(typ.value), shape, int(nb.value))

    def close(self):
        if self._g:
            _lib.load().tb_gguf_close(self._g)
            self._g = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001  (interpreter shutdown)
            pass

    def string(self, key: str):
        v = _lib.load().tb_gguf_get_string(self._g, key.encode())
        return v.decode() if v is not None else None

    def numpy(self, name: str) -> np.ndarray:
        i, typ, shape, nb = self.tensors[name]
        if typ not in _GGUF_NP:
            raise TBError(2, "GgufFile.numpy", f"{name}: ggml type {typ} is not F32/F16/BF16")
        out = np.empty(shape, dtype=_GGUF_NP[typ])
        _io_check(_lib.load().tb_gguf_read_tensor(self._g, i, out.ctypes.data_as(ctypes.c_void_p), nb),
                  "tb_gguf_read_tensor")
        return out

    def to_device(self, name: str, dtype: torch.dtype, device=None) -> torch.Tensor:
        i, typ, shape, nb = self.tensors[name]
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        out = torch.empty(shape, dtype=dtype, device=dev)
        ctx = context(dev)
        check(_lib.load().tb_gguf_upload_tensor(ctx, self._g, i, _DT[dtype], _ptr(out)), "tb_gguf_upload_tensor", ctx)
        return out


def read_slat(path: str):
    """The hr_slat.bin decode input (src/decode_replay.cpp:19-28): (coords int32 [N,3],
    feats float32 [N,32], res)."""
    lib = _lib.load()
    n = ctypes.c_int64()
    res = _lib._i32()
    _io_check(lib.tb_slat_read(str(path).encode(), ctypes.byref(n), ctypes.byref(res), None, None), "tb_slat_read")
    coords = np.empty((n.value, 3), dtype=np.int32)
    feats = np.empty((n.value, 32), dtype=np.float32)
    _io_check(lib.tb_slat_read(str(path).encode(), ctypes.byref(n), ctypes.byref(res),
                               coords.ctypes.data_as(ctypes.c_void_p), feats.ctypes.data_as(ctypes.c_void_p)),
              "tb_slat_read")
    return coords, feats, int(res.value)


# ---- multi-GPU z-slabs (tb_dist_*) --------------------------------------------------------
def zslab_cuts(counts: np.ndarray, z_min: int, world: int) -> np.ndarray:
    """The slab cut of tb_zslab_cuts on the host: counts[i] = voxels of plane z_min + i; returns
    int32 [world + 1] z boundaries (no GPU needed)."""
    c = np.ascontiguousarray(counts, dtype=np.int64)
    cuts = np.empty(world + 1, dtype=np.int32)
    st = _lib.load().tb_zslab_cuts(ctypes.c_void_p(c.ctypes.data), c.size, int(z_min), int(world),
                                   ctypes.c_void_p(cuts.ctypes.data))
    check(st, "tb_zslab_cuts")
    return cuts


def nccl_unique_id() -> bytes:
    """A fresh NCCL unique id (128 bytes) for :class:`Dist`; rank 0 makes it, every rank gets it."""
    buf = (ctypes.c_uint8 * 128)()
    check(_lib.load().tb_nccl_unique_id(ctypes.cast(buf, ctypes.c_void_p)), "tb_nccl_unique_id")
    return bytes(buf)


class Dist:
    """One rank's share of a z-slab sharded voxel set (the tb_dist_* calls of the C ABI).

    ``uid`` is the 128-byte id from :func:`nccl_unique_id` on rank 0, given to every rank; the
    communicator is made by the library (tb_nccl_comm_create). Without ``uid`` nothing is
    exchanged and the caller fills the halo rows (one process driving several slabs). Calls
    enqueue on torch's current stream of ``device``."""

    def __init__(self, device, rank: int, world: int, uid: bytes | None = None, halo_planes: int = 1):
        self.device = torch.device(device)
        self.rank, self.world = rank, world
        lib = _lib.load()
        self.comm = ctypes.c_void_p()
        if uid is not None and world > 1:
            if len(uid) != 128:
                raise ValueError("the NCCL unique id has 128 bytes")
            idb = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
            check(lib.tb_nccl_comm_create(ctypes.cast(idb, ctypes.c_void_p), rank, world, self.device.index,
                                          ctypes.byref(self.comm)), "tb_nccl_comm_create")
        self.h = ctypes.c_void_p()
        ctx = context(self.device)
        check(lib.tb_dist_create(ctx, self.comm, rank, world, ctypes.byref(self.h)), "tb_dist_create", ctx)
        self.slab = None
        self.halo_planes = halo_planes
        self._check(lib.tb_dist_set_halo_planes(self.h, halo_planes), "tb_dist_set_halo_planes")

    def _check(self, st, call):
        if st != _lib.TB_OK:
            d = _lib.load().tb_dist_last_error(self.h)
            raise TBError(st, call, d.decode() if d else "")

    def partition(self, coords: torch.Tensor) -> _lib.ZSlab:
        """Plan this rank's slab of the global voxel set ``coords`` (int32 [N,3] or [N,4])."""
        _need_cuda(coords)
        context(self.device)
        sl = _lib.ZSlab()
        self._check(_lib.load().tb_dist_partition_zslab(self.h, _ptr(coords), coords.shape[0], coords.shape[1],
                                                        ctypes.byref(sl)), "tb_dist_partition_zslab")
        self.slab = sl
        return sl

    def local_rows(self) -> torch.Tensor:
        """Global row ids of the local rows (int32 [n_local])."""
        context(self.device)
        out = torch.empty(max(1, self.slab.n_local), dtype=torch.int32, device=self.device)[: self.slab.n_local]
        self._check(_lib.load().tb_dist_local_rows(self.h, _ptr(out)), "tb_dist_local_rows")
        return out

    def load_coords(self, coords_local: torch.Tensor) -> None:
        _need_cuda(coords_local)
        context(self.device)
        self._check(_lib.load().tb_dist_load_coords(self.h, _ptr(coords_local)), "tb_dist_load_coords")

    def build_map(self) -> None:
        context(self.device)
        self._check(_lib.load().tb_dist_build_map(self.h), "tb_dist_build_map")

    def local_map(self) -> torch.Tensor:
        """The local map ([27 * n_local] int32), a view of the dist-owned buffer (read only)."""
        p = ctypes.c_void_p()
        self._check(_lib.load().tb_dist_local_map(self.h, ctypes.byref(p)), "tb_dist_local_map")
        return _device_view_int32(p.value, 27 * self.slab.n_local, self.device)

    def submconv(self, feats: torch.Tensor, weight: torch.Tensor, bias=None, epi: str = "none", out_dtype=None,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """One conv on the local rows (halo exchange inside); owned rows of the result written."""
        _need_cuda(feats, weight, bias)
        n, ci = feats.shape
        co = weight.shape[0]
        if n != self.slab.n_local or weight.dtype != feats.dtype or weight.numel() != co * 27 * ci:
            raise ValueError("feats must be [n_local, Ci] and weight [Co,27,Ci] of its dtype")
        od = feats.dtype if out_dtype is None else out_dtype
        if out is None:
            out = torch.empty((n, co), dtype=od, device=feats.device)
        context(self.device)
        self._check(_lib.load().tb_dist_submconv(self.h, _ptr(feats), ci, _ptr(weight), _ptr(bias), co,
                                                 _DT[feats.dtype], _DT[od], _EPI[epi], _ptr(out)),
                    "tb_dist_submconv")
        return out

    def exchange(self, feats: torch.Tensor) -> None:
        """Start the halo exchange of ``feats`` ([n_local, C]); the next conv waits for it."""
        _need_cuda(feats)
        if feats.shape[0] != self.slab.n_local or not feats.is_contiguous():
            raise ValueError("feats must be a contiguous [n_local, C] tensor")
        context(self.device)
        self._check(_lib.load().tb_dist_exchange(self.h, _ptr(feats), feats[0].numel() * feats.element_size()),
                    "tb_dist_exchange")

    def local_weight(self, weight: torch.Tensor) -> torch.Tensor:
        """The weight [Co,27,Ci] with its taps in the local map's order (for submconv_grow)."""
        _need_cuda(weight)
        co, _, ci = weight.shape
        out = torch.empty_like(weight)
        context(self.device)
        self._check(_lib.load().tb_dist_local_weight(self.h, _ptr(weight), ci, co, _DT[weight.dtype], _ptr(out)),
                    "tb_dist_local_weight")
        return out

    def submconv_grow(self, grow: int, feats: torch.Tensor, weight_local: torch.Tensor, bias=None,
                      epi: str = "none", out_dtype=None, out: torch.Tensor | None = None) -> torch.Tensor:
        """A conv without exchange on the owned rows and the ``grow`` nearest halo planes per side."""
        _need_cuda(feats, weight_local, bias)
        n, ci = feats.shape
        co = weight_local.shape[0]
        if n != self.slab.n_local or weight_local.dtype != feats.dtype or weight_local.numel() != co * 27 * ci:
            raise ValueError("feats must be [n_local, Ci] and weight_local [Co,27,Ci] of its dtype")
        od = feats.dtype if out_dtype is None else out_dtype
        if out is None:
            out = torch.empty((n, co), dtype=od, device=feats.device)
        context(self.device)
        self._check(_lib.load().tb_dist_submconv_grow(self.h, grow, _ptr(feats), ci, _ptr(weight_local), _ptr(bias),
                                                      co, _DT[feats.dtype], _DT[od], _EPI[epi], _ptr(out)),
                    "tb_dist_submconv_grow")
        return out

    def count_valid_pairs(self) -> int:
        context(self.device)
        v = ctypes.c_int64()
        self._check(_lib.load().tb_dist_count_valid_pairs(self.h, ctypes.byref(v)), "tb_dist_count_valid_pairs")
        return int(v.value)

    def close(self) -> None:
        lib = _lib.load()
        if self.h:
            lib.tb_dist_destroy(self.h)
            self.h = ctypes.c_void_p()
        if self.comm:
            lib.tb_nccl_comm_destroy(self.comm)
            self.comm = ctypes.c_void_p()


def _device_view_int32(ptr: int, n: int, device) -> torch.Tensor:
    """A torch int32 tensor over n elements of library-owned device memory (no copy, not owned)."""
    class _Arr:
        __cuda_array_interface__ = {"shape": (n,), "typestr": "<i4", "data": (ptr, False), "version": 2}
    return torch.as_tensor(_Arr(), device=device)
