"""The sparse decoder UNet (trellis::shape_decode / tex_decode / shape_upsample, the reference's
decode_unet, src/shape_decoder.cpp:79-138) on the device, from a GGUF checkpoint written with
gguf-py (the reference converter's writer), against the oracle composed layer by layer.

The model is small (two stages: widths 64 -> 64 -> 32, three ConvNeXt blocks, two C2S blocks,
from_latent 32 -> 64, output_layer 32 -> 7) but has every layer type of the real one. The oracle
replays the decoder with the subdivision masks the GPU chose (a mask bit can flip where a logit
is within rounding of 0); the stage-0 masks are checked against the oracle's own logits away
from 0. Tolerances (max|d| / max|ref| of the 7 output fields): 1e-3 in the fp32 mode (about a
dozen chained layers of fp32 accumulation), 5e-2 with bf16 weights and activations (weights and
every layer's activations rounded to bf16 on the GPU, not in the oracle)."""
import os
import shutil
import subprocess

import numpy as np
import pytest

import oracle
from conftest import ROOT, max_rel, random_voxels

pytestmark = pytest.mark.gpu

PROGRAM = r"""
#include "trellis_sparse.hpp"
#include <cstdio>
#include <cstdlib>
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
template <class T> void wr(const std::string& name, const T* p, size_t n) {
    FILE* f = std::fopen((g_dir + "/" + name).c_str(), "wb");
    std::fwrite(p, sizeof(T), n, f);
    std::fclose(f);
}

int main(int argc, char** argv) {
    g_dir = argv[1];
    const int n = std::atoi(argv[2]);
    const tb_dtype dt = std::string(argv[3]) == "bf16" ? TB_BF16 : TB_F32;
    try {
        auto c = rd<int>("coords.bin", (size_t)n * 3);
        std::vector<std::array<int, 3>> coords(n);
        for (int i = 0; i < n; ++i) coords[i] = {c[3 * i], c[3 * i + 1], c[3 * i + 2]};
        auto latent = rd<float>("latent.bin", (size_t)n * 32);
        auto m = trellis::GgufModel::load(g_dir + "/model.gguf", 0, dt);
        auto so = trellis::shape_decode(m, latent, coords, 64);
        wr("feats7.out", so.feats7.data(), so.feats7.size());
        wr("coords.out", reinterpret_cast<const int*>(so.coords.data()), so.coords.size() * 3);
        for (size_t s = 0; s < so.subs.size(); ++s)
            wr("subs" + std::to_string(s) + ".out", so.subs[s].data(), so.subs[s].size());
        // the texture decoder grows the same tree from the shape decoder's masks
        auto tex = trellis::tex_decode(m, latent, coords, so.subs);
        wr("tex.out", tex.data(), tex.size());
        auto up = trellis::shape_upsample(m, latent, coords);
        if (up.size() != so.coords.size()) return 3;
        for (size_t i = 0; i < up.size(); ++i)
            if (up[i] != so.coords[i]) return 4;
        std::printf("%zu %zu\n", so.coords.size(), so.subs.size());
    } catch (const std::exception& e) {
        std::fprintf(stderr, "exception: %s\n", e.what());
        return 1;
    }
    return 0;
}
"""

STAGES = [("blocks.0.", 64, 2, 64), ("blocks.1.", 64, 1, 32)]    # prefix, C, ConvNeXt blocks, Cout


def _model(seed):
    rng = np.random.default_rng(seed)
    r = lambda *s, sc=1.0: (rng.standard_normal(s) * sc).astype(np.float32)  # noqa: E731
    w = {"from_latent.weight": r(64, 32, sc=1 / np.sqrt(32)), "from_latent.bias": r(64, sc=0.1)}
    for pre, c, nblk, cout in STAGES:
        for j in range(nblk):
            p = f"{pre}{j}."
            w.update({p + "conv.weight": r(c, 27, c, sc=1 / np.sqrt(27 * c)), p + "conv.bias": r(c, sc=0.1),
                      p + "norm.weight": 1 + r(c, sc=0.1), p + "norm.bias": r(c, sc=0.1),
                      p + "mlp.0.weight": r(4 * c, c, sc=1 / np.sqrt(c)), p + "mlp.0.bias": r(4 * c, sc=0.1),
                      p + "mlp.2.weight": r(c, 4 * c, sc=1 / np.sqrt(4 * c)), p + "mlp.2.bias": r(c, sc=0.1)})
        p = f"{pre}{nblk}."
        w.update({p + "to_subdiv.weight": r(8, c, sc=1 / np.sqrt(c)), p + "to_subdiv.bias": r(8, sc=0.1) - 0.3,
                  p + "norm1.weight": 1 + r(c, sc=0.1), p + "norm1.bias": r(c, sc=0.1),
                  p + "conv1.weight": r(8 * cout, 27, c, sc=1 / np.sqrt(27 * c)), p + "conv1.bias": r(8 * cout, sc=0.1),
                  p + "conv2.weight": r(cout, 27, cout, sc=1 / np.sqrt(27 * cout)), p + "conv2.bias": r(cout, sc=0.1)})
    w["output_layer.weight"] = r(7, 32, sc=1 / np.sqrt(32))
    w["output_layer.bias"] = r(7, sc=0.1)
    return w


def _oracle_decode(w, latent, coords, masks, check_mask0=None):
    h = latent.astype(np.float64) @ w["from_latent.weight"].T.astype(np.float64) + w["from_latent.bias"]
    for s, (pre, c, nblk, cout) in enumerate(STAGES):
        nbr = oracle.build_neighbor_table(coords)
        for j in range(nblk):
            p = f"{pre}{j}."
            conv = oracle.submconv(nbr, h.astype(np.float32), w[p + "conv.weight"], w[p + "conv.bias"])
            y = oracle.layer_norm(conv, w[p + "norm.weight"], w[p + "norm.bias"])
            a = oracle.silu(y @ w[p + "mlp.0.weight"].T.astype(np.float64) + w[p + "mlp.0.bias"])
            h = a @ w[p + "mlp.2.weight"].T.astype(np.float64) + w[p + "mlp.2.bias"] + h
        p = f"{pre}{nblk}."
        if s == 0 and check_mask0 is not None:
            logits = h @ w[p + "to_subdiv.weight"].T.astype(np.float64) + w[p + "to_subdiv.bias"]
            sure = np.abs(logits) > 1e-3
            assert np.array_equal(check_mask0.reshape(-1, 8).astype(bool)[sure], (logits > 0)[sure])
        cw = {k[len(p):]: v for k, v in w.items() if k.startswith(p)}
        o, child, _ = oracle.c2s_block(coords, h.astype(np.float32), cw, cout, ext_mask=masks[s].reshape(-1, 8))
        coords, h = child, o.astype(np.float64)
    y = oracle.layer_norm(h, eps=1e-5)
    return y @ w["output_layer.weight"].T.astype(np.float64) + w["output_layer.bias"], coords


@pytest.mark.parametrize("dtype,tol", [("f32", 1e-3), ("bf16", 5e-2)])
def test_decode_unet_from_gguf(tb, tmp_path, dtype, tol):
    gguf = pytest.importorskip("gguf")
    cxx = shutil.which("g++") or pytest.skip("g++ not found")
    cuda = "/usr/local/cuda"
    from trellis_cpp_b200 import _lib
    n = 300
    coords = random_voxels(n, 16, 7)
    latent = np.random.default_rng(8).standard_normal((n, 32)).astype(np.float32)
    w = _model(9)
    gw = gguf.GGUFWriter(str(tmp_path / "model.gguf"), "trellis2-shape-dec")
    for name, a in w.items():
        gw.add_tensor(name, a)
    gw.write_header_to_file()
    gw.write_kv_data_to_file()
    gw.write_tensors_to_file()
    gw.close()
    coords.astype(np.int32).tofile(tmp_path / "coords.bin")
    latent.tofile(tmp_path / "latent.bin")
    src = tmp_path / "decode.cpp"
    src.write_text(PROGRAM)
    exe = tmp_path / "decode"
    libdir = os.path.dirname(_lib.LIB_PATH)
    b = subprocess.run([cxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"), "-I", cuda + "/include",
                        str(src), "-o", str(exe), "-L", libdir, "-ltb_sparse", "-Wl,-rpath," + libdir,
                        "-L", cuda + "/lib64", "-lcudart", "-Wl,-rpath," + cuda + "/lib64"],
                       capture_output=True, text=True)
    assert b.returncode == 0, b.stderr
    r = subprocess.run([str(exe), str(tmp_path), str(n), dtype], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    m_final, nsubs = map(int, r.stdout.split())
    assert nsubs == len(STAGES)
    subs = [np.fromfile(tmp_path / f"subs{s}.out", dtype=np.uint8) for s in range(nsubs)]
    feats7 = np.fromfile(tmp_path / "feats7.out", dtype=np.float32).reshape(m_final, 7)
    out_coords = np.fromfile(tmp_path / "coords.out", dtype=np.int32).reshape(m_final, 3)
    ref, ref_coords = _oracle_decode(w, latent, coords, subs, check_mask0=subs[0] if dtype == "f32" else None)
    assert m_final > n and np.array_equal(out_coords, ref_coords)
    assert max_rel(feats7, ref) < tol
    tex = np.fromfile(tmp_path / "tex.out", dtype=np.float32).reshape(m_final, 7)
    assert np.array_equal(tex, feats7)     # same weights, same masks: the same decode
