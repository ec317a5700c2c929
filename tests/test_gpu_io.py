"""GGUF tensors uploaded to the device (tb_gguf_upload_tensor) and used by the kernels.

Conversions on upload must equal torch's round-to-nearest-even conversions; a ConvNeXt block whose
weights come from a GGUF file written with the reference's conversion policy (tools/convert.py:
weights F16, 1-D parameters F32) must give exactly the result of the same weights passed
directly."""
import numpy as np
import pytest
import torch

from conftest import random_voxels

pytestmark = pytest.mark.gpu
gguf = pytest.importorskip("gguf")


def _write(path, tensors):
    w = gguf.GGUFWriter(str(path), "trellis2-shape-dec")
    for name, a in tensors.items():
        if a.dtype == np.uint16:
            w.add_tensor(name, a, raw_dtype=gguf.GGMLQuantizationType.BF16)
        else:
            w.add_tensor(name, a)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def test_upload_conversions(tb, tmp_path):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(1)
    a32 = (rng.standard_normal((7, 33)) * 100).astype(np.float32)
    a16 = rng.standard_normal((5, 40)).astype(np.float16)
    abf = torch.from_numpy(rng.standard_normal((3, 24)).astype(np.float32)).bfloat16()
    _write(tmp_path / "c.gguf", {"a32": a32, "a16": a16, "abf": abf.view(torch.int16).numpy().view(np.uint16)})
    f = ops.GgufFile(tmp_path / "c.gguf")
    t32 = torch.from_numpy(a32)
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        assert torch.equal(f.to_device("a32", dt).cpu(), t32.to(dt))
        assert torch.equal(f.to_device("a16", dt).cpu(), torch.from_numpy(a16).to(dt))
        assert torch.equal(f.to_device("abf", dt).cpu(), abf.to(dt))
    f.close()


def test_convnext_block_from_gguf(tb, tmp_path):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(4)
    n, c = 4000, 64
    t = {
        "blk.conv.weight": (rng.standard_normal((c, 27, c)) / np.sqrt(27 * c)).astype(np.float16),
        "blk.conv.bias": (0.1 * rng.standard_normal(c)).astype(np.float32),
        "blk.norm.weight": (1 + 0.1 * rng.standard_normal(c)).astype(np.float32),
        "blk.norm.bias": (0.1 * rng.standard_normal(c)).astype(np.float32),
        "blk.mlp.0.weight": (rng.standard_normal((4 * c, c)) / np.sqrt(c)).astype(np.float16),
        "blk.mlp.0.bias": (0.1 * rng.standard_normal(4 * c)).astype(np.float32),
        "blk.mlp.2.weight": (rng.standard_normal((c, 4 * c)) / np.sqrt(4 * c)).astype(np.float16),
        "blk.mlp.2.bias": (0.1 * rng.standard_normal(c)).astype(np.float32),
    }
    _write(tmp_path / "b.gguf", t)
    f = ops.GgufFile(tmp_path / "b.gguf")
    bf = torch.bfloat16
    g = {k: f.to_device(k, bf if v.ndim >= 2 else torch.float32) for k, v in t.items()}
    d = {k: torch.from_numpy(v.astype(np.float32)).cuda().to(bf if v.ndim >= 2 else torch.float32)
         for k, v in t.items()}
    coords = torch.from_numpy(random_voxels(n, 30, 4)).cuda()
    nbr = ops.build_neighbor_table(coords)
    x = torch.randn((n, c), device="cuda").to(bf)

    def run(p):
        return ops.sparse_convnext(x, nbr, p["blk.conv.weight"], p["blk.conv.bias"], p["blk.norm.weight"],
                                   p["blk.norm.bias"], p["blk.mlp.0.weight"], p["blk.mlp.0.bias"],
                                   p["blk.mlp.2.weight"], p["blk.mlp.2.bias"], out_dtype=torch.float32)
    a, b = run(g), run(d)
    ops.check_device()
    assert torch.equal(a, b)
    f.close()
