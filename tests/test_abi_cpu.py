"""CPU-only checks of the C-ABI library: it loads without a GPU and exports every symbol
include/tb_sparse.h declares. No compute call is made here."""
import os
import re
import shutil
import subprocess

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


C_PROGRAM = r"""
#include "tb_sparse.h"
#include <stdio.h>
#include <string.h>

int main(void) {
    /* the declarations are plain C; taking the entry points' addresses links them */
    tb_status (*mesh)(tb_ctx*, const int32_t*, int64_t, int, const float*, int, float*, int32_t*, int64_t,
                      int64_t*) = tb_dual_grid_mesh;
    tb_status (*conv)(tb_ctx*, const int32_t*, int64_t, const void*, int, const void*, const float*, int,
                      tb_dtype, tb_dtype, tb_epilogue, void*) = tb_submconv;
    tb_c2s_params p;
    memset(&p, 0, sizeof p);
    if (!mesh || !conv || p.conv1_w) return 2;
    printf("%s|%s\n", tb_status_string(TB_OK), tb_version());
    return 0;
}
"""


def test_header_is_plain_c_and_links(tb, tmp_path):
    # an FFI generator or a C caller includes tb_sparse.h as C99 and links libtb_sparse.so
    cc = shutil.which("gcc") or pytest.skip("gcc not found")
    from trellis_cpp_b200 import _lib
    libdir = os.path.dirname(_lib.LIB_PATH)
    (tmp_path / "abi.c").write_text(C_PROGRAM)
    b = subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(tmp_path / "abi.c"), "-o", str(tmp_path / "abi"), "-L", libdir, "-ltb_sparse",
                        "-Wl,-rpath," + libdir], capture_output=True, text=True)
    assert b.returncode == 0, b.stderr
    r = subprocess.run([str(tmp_path / "abi")], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    status, version = r.stdout.strip().split("|")
    assert status == "ok" and "sm_100a" in version


CXX_PROGRAM = r"""
#include "trellis_sparse.hpp"
#include <cstdio>

// Every host-mirror entry point, referenced so that the link resolves it; run() is never
// called on a box without a GPU (main only runs it with an argument).
static int run() {
    std::vector<std::array<int, 3>> c{{0, 0, 0}};
    std::vector<float> f(64, 0.f);
    auto nbr = trellis::build_neighbor_table(c);
    trellis::ConvWeights cw{};
    auto y = trellis::sparse_submconv(cw, f, nbr, 1);
    trellis::ConvNeXtWeights nw{};
    auto z = trellis::sparse_convnext(nw, f, nbr, 1);
    auto sd = trellis::subdivide(c, std::vector<uint8_t>(8, 1));
    trellis::C2SWeights c2{};
    auto up = trellis::sparse_c2s(c2, f, 64, c, 32);
    auto m = trellis::GgufModel::load("model.gguf");
    auto sl = trellis::read_slat("hr_slat.bin");
    auto so = trellis::shape_decode(m, sl.feats, sl.coords);
    auto gc = trellis::shape_upsample(m, sl.feats, sl.coords);
    auto tx = trellis::tex_decode(m, sl.feats, sl.coords, so.subs);
    trellis::Mesh mesh = trellis::dual_grid_to_mesh(so);
    return (int)(y.size() + z.size() + sd.coords.size() + up.feats.size() + gc.size() + tx.size()) + mesh.F();
}

int main(int argc, char**) {
    if (argc > 1) return run();
    std::printf("%s\n", tb_version());
    return 0;
}
"""


def test_cxx_mirror_header_compiles_and_links(tb, tmp_path):
    cxx = shutil.which("g++") or pytest.skip("g++ not found")
    from trellis_cpp_b200 import _lib
    libdir = os.path.dirname(_lib.LIB_PATH)
    (tmp_path / "mirror.cpp").write_text(CXX_PROGRAM)
    b = subprocess.run([cxx, "-std=c++17", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        str(tmp_path / "mirror.cpp"), "-o", str(tmp_path / "mirror"), "-L", libdir, "-ltb_sparse",
                        "-Wl,-rpath," + libdir], capture_output=True, text=True)
    assert b.returncode == 0, b.stderr
    r = subprocess.run([str(tmp_path / "mirror")], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "sm_100a" in r.stdout, r.stdout + r.stderr
