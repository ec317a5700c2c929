"""The C++ host mirror (include/trellis_sparse.hpp: the reference's include/sparse.h names) on the
GPU: a small C++ program built against the header and libtb_sparse.so runs
build_neighbor_table, sparse_submconv, sparse_convnext and sparse_c2s on the golden inputs of
the reference's torch restatements (fp32 mode), once with weights it uploads itself and once
with weights loaded by GgufModel from GGUF files written by gguf-py (the reference's converter's
writer), and reads an hr_slat.bin dump; the outputs are compared here (maps and child
coordinates exactly, features at max|d|/max|ref| < 1e-4)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from conftest import ROOT, max_rel

pytestmark = pytest.mark.gpu

PROGRAM = r"""
#include "trellis_sparse.hpp"
#include <cuda_runtime.h>
#include <cstdio>
#include <cstdlib>
#include <stdexcept>
#include <string>
#include <vector>

static std::string g_dir;
template <class T> std::vector<T> rd(const char* name, size_t n) {
    std::vector<T> v(n);
    FILE* f = std::fopen((g_dir + "/" + name).c_str(), "rb");
    if (!f || std::fread(v.data(), sizeof(T), n, f) != n) { std::fprintf(stderr, "read %s\n", name); std::exit(2); }
    std::fclose(f);
    return v;
}
template <class T> void wr(const char* name, const T* p, size_t n) {
    FILE* f = std::fopen((g_dir + "/" + name).c_str(), "wb");
    std::fwrite(p, sizeof(T), n, f);
    std::fclose(f);
}
template <class T> T* dev(const std::vector<T>& v) {
    T* p = nullptr;
    if (cudaMalloc(&p, v.size() * sizeof(T) + 16) != cudaSuccess) std::exit(3);
    cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
    return p;
}
static std::vector<std::array<int, 3>> as_coords(const std::vector<int>& c) {
    std::vector<std::array<int, 3>> r(c.size() / 3);
    for (size_t i = 0; i < r.size(); ++i) r[i] = {c[3 * i], c[3 * i + 1], c[3 * i + 2]};
    return r;
}

int main(int argc, char** argv) {
    g_dir = argv[1];
    const int n = std::atoi(argv[2]), c = std::atoi(argv[3]), n2 = std::atoi(argv[4]), cin = std::atoi(argv[5]),
              cout = std::atoi(argv[6]);
    try {
        // ---- conv + ConvNeXt block on the submconv golden case
        auto coords = as_coords(rd<int>("coords.bin", (size_t)n * 3));
        auto feats = rd<float>("feats.bin", (size_t)n * c);
        auto nbr = trellis::build_neighbor_table(coords);
        wr("nbr.out", nbr.data(), nbr.size());
        trellis::ConvWeights cw;
        cw.weight = dev(rd<float>("conv_w.bin", (size_t)c * 27 * c));
        cw.bias = dev(rd<float>("conv_b.bin", c));
        cw.ci = cw.co = c;
        cw.dtype = TB_F32;
        auto conv = trellis::sparse_submconv(cw, feats, nbr, n);
        wr("conv.out", conv.data(), conv.size());
        trellis::ConvNeXtWeights xw;
        xw.conv = cw;
        xw.norm_w = dev(rd<float>("norm_w.bin", c));
        xw.norm_b = dev(rd<float>("norm_b.bin", c));
        xw.mlp0_w = dev(rd<float>("mlp0_w.bin", (size_t)4 * c * c));
        xw.mlp0_b = dev(rd<float>("mlp0_b.bin", (size_t)4 * c));
        xw.mlp2_w = dev(rd<float>("mlp2_w.bin", (size_t)4 * c * c));
        xw.mlp2_b = dev(rd<float>("mlp2_b.bin", c));
        auto blk = trellis::sparse_convnext(xw, feats, nbr, n);
        wr("block.out", blk.data(), blk.size());
        // ---- the C2S block on the c2s golden case, with the reference's mask
        auto coords2 = as_coords(rd<int>("c2s_coords.bin", (size_t)n2 * 3));
        auto feats2 = rd<float>("c2s_feats.bin", (size_t)n2 * cin);
        auto mask = rd<uint8_t>("c2s_mask.bin", (size_t)n2 * 8);
        trellis::C2SWeights w;
        w.dtype = TB_F32;
        w.p.to_subdiv_w = dev(rd<float>("sd_w.bin", (size_t)8 * cin));
        w.p.to_subdiv_b = dev(rd<float>("sd_b.bin", 8));
        w.p.norm1_w = dev(rd<float>("n1_w.bin", cin));
        w.p.norm1_b = dev(rd<float>("n1_b.bin", cin));
        w.p.conv1_w = dev(rd<float>("c1_w.bin", (size_t)8 * cout * 27 * cin));
        w.p.conv1_b = dev(rd<float>("c1_b.bin", (size_t)8 * cout));
        w.p.conv2_w = dev(rd<float>("c2_w.bin", (size_t)cout * 27 * cout));
        w.p.conv2_b = dev(rd<float>("c2_b.bin", cout));
        auto r = trellis::sparse_c2s(w, feats2, cin, coords2, cout, &mask);
        wr("c2s_feats.out", r.feats.data(), r.feats.size());
        wr("c2s_coords.out", reinterpret_cast<const int*>(r.coords.data()), r.coords.size() * 3);
        wr("c2s_mask.out", r.subdiv.data(), r.subdiv.size());
        auto r2 = trellis::sparse_c2s(w, feats2, cin, coords2, cout, nullptr);   // mask from to_subdiv
        wr("c2s_mask2.out", r2.subdiv.data(), r2.subdiv.size());
        // ---- the same blocks with weights from GGUF checkpoints, looked up by prefix
        {
            auto m = trellis::GgufModel::load(g_dir + "/model.gguf", 0, TB_F32);
            if (m.arch != "trellis2-shape-dec" || m.config_json.empty()) return 5;
            auto blk2 = trellis::sparse_convnext(m.convnext("blk"), feats, nbr, n);
            wr("block_gguf.out", blk2.data(), blk2.size());
            auto r3 = trellis::sparse_c2s(m.c2s("up"), feats2, cin, coords2, cout, &mask);
            wr("c2s_gguf.out", r3.feats.data(), r3.feats.size());
            bool threw2 = false;
            try {
                m.conv("no.such.block");
            } catch (const std::runtime_error&) {
                threw2 = true;
            }
            if (!threw2) return 6;
        }
        auto slat = trellis::read_slat(g_dir + "/hr_slat.bin");
        wr("slat_coords.out", reinterpret_cast<const int*>(slat.coords.data()), slat.coords.size() * 3);
        wr("slat_feats.out", slat.feats.data(), slat.feats.size());
        if (slat.res != 512) return 7;
        // errors throw like the reference
        bool threw = false;
        try {
            trellis::sparse_c2s(w, feats2, cin + 8, coords2, cout, &mask);
        } catch (const std::runtime_error&) {
            threw = true;
        }
        if (!threw) return 4;
    } catch (const std::exception& e) {
        std::fprintf(stderr, "exception: %s\n", e.what());
        return 1;
    }
    std::printf("ok\n");
    return 0;
}
"""


def _cuda_home():
    for p in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if p and os.path.exists(os.path.join(p, "include", "cuda_runtime.h")):
            return p
    pytest.skip("CUDA headers not found")


def test_cxx_mirror_on_golden_cases(tb, golden, tmp_path):
    from trellis_cpp_b200 import _lib
    cuda = _cuda_home()
    cxx = shutil.which("g++") or pytest.skip("g++ not found")
    g, g2 = golden["submconv"], golden["c2s"]
    n, c = g["feats"].shape
    n2, cin = g2["feats"].shape
    cout = 16
    files = {
        "coords.bin": g["coords"], "feats.bin": g["feats"], "conv_w.bin": g["weight"], "conv_b.bin": g["bias"],
        "norm_w.bin": g["norm.weight"], "norm_b.bin": g["norm.bias"], "mlp0_w.bin": g["mlp.0.weight"],
        "mlp0_b.bin": g["mlp.0.bias"], "mlp2_w.bin": g["mlp.2.weight"], "mlp2_b.bin": g["mlp.2.bias"],
        "c2s_coords.bin": g2["coords"], "c2s_feats.bin": g2["feats"], "c2s_mask.bin": g2["mask"],
        "sd_w.bin": g2["to_subdiv.weight"], "sd_b.bin": g2["to_subdiv.bias"], "n1_w.bin": g2["norm1.weight"],
        "n1_b.bin": g2["norm1.bias"], "c1_w.bin": g2["conv1.weight"], "c1_b.bin": g2["conv1.bias"],
        "c2_w.bin": g2["conv2.weight"], "c2_b.bin": g2["conv2.bias"],
    }
    for name, a in files.items():
        np.ascontiguousarray(a).tofile(tmp_path / name)
    # a GGUF checkpoint holding both blocks under the reference's tensor names (fp32 throughout,
    # as tools/convert.py writes with FORCE_F32=1)
    gguf = pytest.importorskip("gguf")
    gw = gguf.GGUFWriter(str(tmp_path / "model.gguf"), "trellis2-shape-dec")
    gw.add_string("trellis.config_json", "{}")
    c2 = lambda a: np.ascontiguousarray(a.reshape(a.shape[0], 27, -1), dtype=np.float32)  # noqa: E731
    for name, a in (("blk.conv.weight", c2(g["weight"])), ("blk.conv.bias", g["bias"]),
                    ("blk.norm.weight", g["norm.weight"]), ("blk.norm.bias", g["norm.bias"]),
                    ("blk.mlp.0.weight", g["mlp.0.weight"]), ("blk.mlp.0.bias", g["mlp.0.bias"]),
                    ("blk.mlp.2.weight", g["mlp.2.weight"]), ("blk.mlp.2.bias", g["mlp.2.bias"]),
                    ("up.to_subdiv.weight", g2["to_subdiv.weight"]), ("up.to_subdiv.bias", g2["to_subdiv.bias"]),
                    ("up.norm1.weight", g2["norm1.weight"]), ("up.norm1.bias", g2["norm1.bias"]),
                    ("up.conv1.weight", c2(g2["conv1.weight"])), ("up.conv1.bias", g2["conv1.bias"]),
                    ("up.conv2.weight", c2(g2["conv2.weight"])), ("up.conv2.bias", g2["conv2.bias"])):
        gw.add_tensor(name, np.ascontiguousarray(a, dtype=np.float32))
    gw.write_header_to_file()
    gw.write_kv_data_to_file()
    gw.write_tensors_to_file()
    gw.close()
    rng = np.random.default_rng(5)
    slat_c = rng.integers(0, 512, (300, 3)).astype(np.int32)
    slat_f = rng.standard_normal((300, 32)).astype(np.float32)
    with open(tmp_path / "hr_slat.bin", "wb") as fh:
        fh.write(np.array([300, 512], dtype=np.int32).tobytes() + slat_c.tobytes() + slat_f.tobytes())
    src = tmp_path / "mirror.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "mirror"
    libdir = os.path.dirname(_lib.LIB_PATH)
    b = subprocess.run([cxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), "-I",
                        os.path.join(cuda, "include"), str(src), "-o", str(exe), "-L", libdir, "-ltb_sparse",
                        "-Wl,-rpath," + libdir, "-L", os.path.join(cuda, "lib64"), "-lcudart",
                        "-Wl,-rpath," + os.path.join(cuda, "lib64")], capture_output=True, text=True)
    assert b.returncode == 0, b.stderr
    r = subprocess.run([str(exe), str(tmp_path), str(n), str(c), str(n2), str(cin), str(cout)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    nbr = np.fromfile(tmp_path / "nbr.out", dtype=np.int32)
    assert np.array_equal(nbr, oracle.build_neighbor_table(g["coords"]).reshape(-1))
    conv = np.fromfile(tmp_path / "conv.out", dtype=np.float32).reshape(n, c)
    assert max_rel(conv, g["conv_out"]) < 1e-4
    blk = np.fromfile(tmp_path / "block.out", dtype=np.float32).reshape(n, c)
    assert max_rel(blk, g["block_out"]) < 1e-4
    child = np.fromfile(tmp_path / "c2s_coords.out", dtype=np.int32).reshape(-1, 3)
    assert np.array_equal(child, g2["new_coords"])
    out = np.fromfile(tmp_path / "c2s_feats.out", dtype=np.float32).reshape(-1, cout)
    assert max_rel(out, g2["out"]) < 1e-4
    assert np.array_equal(np.fromfile(tmp_path / "c2s_mask.out", dtype=np.uint8).reshape(n2, 8), g2["mask"])
    assert max_rel(np.fromfile(tmp_path / "block_gguf.out", dtype=np.float32).reshape(n, c), g["block_out"]) < 1e-4
    out_g = np.fromfile(tmp_path / "c2s_gguf.out", dtype=np.float32).reshape(-1, cout)
    assert max_rel(out_g, g2["out"]) < 1e-4
    assert np.array_equal(np.fromfile(tmp_path / "slat_coords.out", dtype=np.int32).reshape(-1, 3), slat_c)
    assert np.array_equal(np.fromfile(tmp_path / "slat_feats.out", dtype=np.float32).reshape(-1, 32), slat_f)
    sure = np.abs(g2["subdiv"]) > 1e-5
    mask2 = np.fromfile(tmp_path / "c2s_mask2.out", dtype=np.uint8).reshape(n2, 8)
    assert np.array_equal(mask2[sure], g2["mask"][sure])
