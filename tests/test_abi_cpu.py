"""CPU-only checks of the C-ABI library: it loads without a GPU and exports every symbol
include/tb_sparse.h declares. No compute call is made here."""
import os
import re

import pytest

from conftest import ROOT


def _declared_symbols():
    src = open(os.path.join(ROOT, "include", "tb_sparse.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(tb_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_entry_points():
    syms = _declared_symbols()
    for s in ("tb_build_neighbor_map", "tb_submconv", "tb_subdivide", "tb_c2s_gather", "tb_bias_act",
              "tb_submconv_stack_host", "tb_ctx_create", "tb_ctx_destroy", "tb_convnext_tail",
              "tb_sparse_convnext", "tb_sparse_c2s"):
        assert s in syms


def test_library_exports_every_declared_symbol(tb):
    from trellis_cpp_b200 import _lib
    lib = _lib.load()
    for s in _declared_symbols():
        assert hasattr(lib, s), f"{s} declared in tb_sparse.h but not exported"
    assert set(_declared_symbols()) <= set(_lib.SIGNATURES)


def test_status_strings_and_version(tb):
    from trellis_cpp_b200 import _lib
    lib = _lib.load()
    assert lib.tb_status_string(0) == b"ok"
    assert lib.tb_status_string(2) == b"unsupported configuration"
    assert b"sm_100a" in lib.tb_version()


def test_cxx_mirror_header_matches_reference_names():
    # the C++ mirror keeps the reference's host names (include/sparse.h:14-35)
    src = open(os.path.join(ROOT, "include", "trellis_sparse.hpp")).read()
    for name in ("build_neighbor_table", "sparse_submconv", "subdivide", "namespace trellis"):
        assert name in src
