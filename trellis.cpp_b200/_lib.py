"""ctypes binding of libtb_sparse.so (the C ABI declared in include/tb_sparse.h).

Loading the library needs no GPU; every compute entry point does. There is no fallback:
if the library is missing, loading raises.
"""
from __future__ import annotations

import ctypes
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libtb_sparse.so")

TB_OK = 0
STATUS = {0: "TB_OK", 1: "TB_ERR_INVALID_ARG", 2: "TB_ERR_UNSUPPORTED", 3: "TB_ERR_CUDA",
          4: "TB_ERR_OUT_OF_MEMORY", 5: "TB_ERR_DEVICE", 6: "TB_ERR_TOO_LARGE"}
TB_F32, TB_F16, TB_BF16 = 0, 1, 2
TB_EPI_NONE, TB_EPI_SILU = 0, 1
TB_CONV_AUTO, TB_CONV_GATHER, TB_CONV_BRICK, TB_CONV_PAIR = 0, 1, 2, 3

# Every symbol include/tb_sparse.h declares, with (restype, argtypes).
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_int = ctypes.c_int
_st = ctypes.c_int


class ConvLayer(ctypes.Structure):
    """tb_conv_layer (include/tb_sparse.h)."""
    _fields_ = [("weight", _vp), ("bias", _vp), ("ci", _int), ("co", _int), ("epi", _int)]


class C2SParams(ctypes.Structure):
    """tb_c2s_params (include/tb_sparse.h)."""
    _fields_ = [("to_subdiv_w", _vp), ("to_subdiv_b", _vp), ("norm1_w", _vp), ("norm1_b", _vp),
                ("conv1_w", _vp), ("conv1_b", _vp), ("conv2_w", _vp), ("conv2_b", _vp)]


class ZSlab(ctypes.Structure):
    """tb_zslab (include/tb_sparse.h)."""
    _fields_ = [("z_lo", _i32), ("z_hi", _i32), ("n_local", _i64), ("n_owned", _i64), ("owned_begin", _i64),
                ("n_halo_lo", _i64), ("n_halo_hi", _i64), ("n_edge_lo", _i64), ("n_edge_hi", _i64)]


SIGNATURES = {
    "tb_status_string": (ctypes.c_char_p, [_st]),
    "tb_version": (ctypes.c_char_p, []),
    "tb_ctx_create": (_st, [_int, _vp, ctypes.POINTER(_vp)]),
    "tb_ctx_destroy": (_st, [_vp]),
    "tb_ctx_set_stream": (_st, [_vp, _vp]),
    "tb_ctx_last_error": (ctypes.c_char_p, [_vp]),
    "tb_ctx_check_device": (_st, [_vp]),
    "tb_ctx_set_conv_path": (_st, [_vp, _int]),
    "tb_build_neighbor_map": (_st, [_vp, _vp, _i64, _int, _vp]),
    "tb_build_neighbor_map_noalloc": (_st, [_vp, _vp, _i64, _int, _vp]),
    "tb_count_valid_pairs": (_st, [_vp, _vp, _i64, ctypes.POINTER(_i64)]),
    "tb_submconv": (_st, [_vp, _vp, _i64, _vp, _int, _vp, _vp, _int, _int, _int, _int, _vp]),
    "tb_submconv_range": (_st, [_vp, _vp, _i64, _i64, _i64, _vp, _int, _vp, _vp, _int, _int, _int, _int, _vp]),
    "tb_sort_rows": (_st, [_vp, _vp, _i64, _int, _vp]),
    "tb_subdivide": (_st, [_vp, _vp, _i64, _int, _vp, _vp, _vp, _vp, _i64, ctypes.POINTER(_i64)]),
    "tb_c2s_gather": (_st, [_vp, _vp, _vp, _i64, _int, _int, _vp]),
    "tb_dual_grid_mesh": (_st, [_vp, _vp, _i64, _int, _vp, _int, _vp, _vp, _i64, ctypes.POINTER(_i64)]),
    "tb_bias_act": (_st, [_vp, _vp, _i64, _int, _vp, _int, _int]),
    "tb_submconv_stack_host": (_st, [_vp, _vp, _i64, _int, _vp, ctypes.POINTER(ConvLayer), _int, _int,
                                     _int, _vp]),
    "tb_zslab_counts": (_st, [_vp, _vp, _i64, _int, _i32, _i32, _vp]),
    "tb_gather_rows": (_st, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "tb_scatter_rows": (_st, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "tb_convnext_tail": (_st, [_vp, _i64, _int, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _vp]),
    "tb_sparse_convnext": (_st, [_vp, _vp, _i64, _vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int,
                                 _vp]),
    "tb_linear": (_st, [_vp, _i64, _int, _int, _vp, _vp, _vp, _vp, _int, _int, _int, _int, _vp]),
    "tb_layer_norm": (_st, [_vp, _vp, _int, _i64, _int, _vp, _vp, ctypes.c_float, _int, _int, _vp]),
    "tb_gguf_open": (_st, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "tb_gguf_close": (None, [_vp]),
    "tb_gguf_n_tensors": (_i64, [_vp]),
    "tb_gguf_find_tensor": (_i64, [_vp, ctypes.c_char_p]),
    "tb_gguf_tensor_info": (_st, [_vp, _i64, ctypes.POINTER(ctypes.c_char_p), ctypes.POINTER(_i32),
                                  ctypes.POINTER(_i32), ctypes.POINTER(_i64), ctypes.POINTER(ctypes.c_uint64)]),
    "tb_gguf_get_string": (ctypes.c_char_p, [_vp, ctypes.c_char_p]),
    "tb_gguf_read_tensor": (_st, [_vp, _i64, _vp, ctypes.c_uint64]),
    "tb_gguf_upload_tensor": (_st, [_vp, _vp, _i64, _int, _vp]),
    "tb_slat_read": (_st, [ctypes.c_char_p, ctypes.POINTER(_i64), ctypes.POINTER(_i32), _vp, _vp]),
    "tb_io_last_error": (ctypes.c_char_p, []),
    "tb_sparse_c2s": (_st, [_vp, _vp, _i64, _int, _vp, _int, _int, ctypes.POINTER(C2SParams), _vp, _int, _int,
                            _i64, _vp, _vp, _vp, ctypes.POINTER(_i64)]),
    "tb_nccl_unique_id": (_st, [_vp]),
    "tb_nccl_comm_create": (_st, [_vp, _int, _int, _int, ctypes.POINTER(_vp)]),
    "tb_nccl_comm_destroy": (_st, [_vp]),
    "tb_dist_create": (_st, [_vp, _vp, _int, _int, ctypes.POINTER(_vp)]),
    "tb_dist_destroy": (_st, [_vp]),
    "tb_dist_last_error": (ctypes.c_char_p, [_vp]),
    "tb_dist_partition_zslab": (_st, [_vp, _vp, _i64, _int, ctypes.POINTER(ZSlab)]),
    "tb_dist_local_rows": (_st, [_vp, _vp]),
    "tb_dist_load_coords": (_st, [_vp, _vp]),
    "tb_dist_build_map": (_st, [_vp]),
    "tb_dist_local_map": (_st, [_vp, ctypes.POINTER(_vp)]),
    "tb_dist_submconv": (_st, [_vp, _vp, _int, _vp, _vp, _int, _int, _int, _int, _vp]),
    "tb_dist_count_valid_pairs": (_st, [_vp, ctypes.POINTER(_i64)]),
    "tb_dist_set_halo_planes": (_st, [_vp, _int]),
    "tb_dist_exchange": (_st, [_vp, _vp, _i64]),
    "tb_dist_local_weight": (_st, [_vp, _vp, _int, _int, _int, _vp]),
    "tb_dist_submconv_grow": (_st, [_vp, _int, _vp, _int, _vp, _vp, _int, _int, _int, _int, _vp]),
    "tb_zslab_cuts": (_st, [_vp, _i32, _i32, _int, _vp]),
}

_lib = None


def load():
    """Load the library (raises OSError/FileNotFoundError when it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python trellis.cpp_b200/build.py` "
                "(or __graft_entry__.build()); there is no CPU fallback")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


class TBError(RuntimeError):
    def __init__(self, status: int, call: str, detail: str = ""):
        self.status = status
        super().__init__(f"{call} -> {STATUS.get(status, status)}" + (f": {detail}" if detail else ""))


def check(status: int, call: str, ctx=None):
    if status != TB_OK:
        detail = ""
        if ctx is not None:
            d = load().tb_ctx_last_error(ctx)
            detail = d.decode() if d else ""
        raise TBError(status, call, detail)
