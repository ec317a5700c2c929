"""GPU SparseResBlockC2S3d (tb_sparse_c2s, src/sparse.cpp:172-336) vs the golden output of the
reference's torch restatement and vs the CPU oracle.

Tolerances (max|d| / max|ref|): 1e-4 in the fp32 mode against the golden output; 1e-2 with
bf16/f16 operands against the fp64 oracle on the unrounded data (the path's stated tolerance for
16-bit operands). Child coordinates and masks are compared exactly; a mask computed from the
to_subdiv logits may differ only where the logit is within fp32 rounding of 0."""
import numpy as np
import pytest
import torch

import oracle
from conftest import max_rel, random_voxels, round_to

pytestmark = pytest.mark.gpu

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _cuda(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(dt)


def _golden_params(g, dt=torch.float32):
    p = {k: _cuda(g[k]) for k in ("to_subdiv.weight", "to_subdiv.bias", "norm1.weight", "norm1.bias",
                                  "conv1.bias", "conv2.bias")}
    p["conv1.weight"] = _cuda(g["conv1.weight"].reshape(g["conv1.weight"].shape[0], 27, -1), dt)
    p["conv2.weight"] = _cuda(g["conv2.weight"].reshape(g["conv2.weight"].shape[0], 27, -1), dt)
    return p


def test_golden_block_fp32_external_mask(tb, golden):
    from trellis_cpp_b200 import ops
    g = golden["c2s"]
    coords = torch.from_numpy(g["coords"]).cuda()
    out, child, mask = ops.sparse_c2s(coords, _cuda(g["feats"]), _golden_params(g), cout=16,
                                      ext_mask=torch.from_numpy(g["mask"]).cuda())
    ops.check_device()
    assert np.array_equal(child.cpu().numpy(), g["new_coords"])
    assert np.array_equal(mask.cpu().numpy(), g["mask"])
    assert max_rel(out.cpu().numpy(), g["out"]) < 1e-4


def test_golden_block_fp32_mask_from_logits(tb, golden):
    from trellis_cpp_b200 import ops
    g = golden["c2s"]
    sure = np.abs(g["subdiv"]) > 1e-5
    out, child, mask = ops.sparse_c2s(torch.from_numpy(g["coords"]).cuda(), _cuda(g["feats"]), _golden_params(g),
                                      cout=16)
    ops.check_device()
    mask = mask.cpu().numpy()
    assert np.array_equal(mask[sure], g["mask"][sure])
    if np.array_equal(mask, g["mask"]):
        assert np.array_equal(child.cpu().numpy(), g["new_coords"])
        assert max_rel(out.cpu().numpy(), g["out"]) < 1e-4


def _random_case(n, cin, cout, dtype, seed, box=40):
    rng = np.random.default_rng(seed)
    coords = random_voxels(n, box, seed)
    feats = round_to(rng.standard_normal((n, cin)).astype(np.float32), dtype)
    w = {
        "to_subdiv.weight": (rng.standard_normal((8, cin)) / np.sqrt(cin)).astype(np.float32),
        "to_subdiv.bias": (0.1 * rng.standard_normal(8)).astype(np.float32),
        "norm1.weight": (1 + 0.1 * rng.standard_normal(cin)).astype(np.float32),
        "norm1.bias": (0.1 * rng.standard_normal(cin)).astype(np.float32),
        "conv1.weight": round_to((rng.standard_normal((8 * cout, 27, cin)) / np.sqrt(27 * cin)).astype(np.float32),
                                 dtype),
        "conv1.bias": (0.1 * rng.standard_normal(8 * cout)).astype(np.float32),
        "conv2.weight": round_to((rng.standard_normal((cout, 27, cout)) / np.sqrt(27 * cout)).astype(np.float32),
                                 dtype),
        "conv2.bias": (0.1 * rng.standard_normal(cout)).astype(np.float32),
    }
    return coords, feats, w


def _params(w, dt):
    return {k: _cuda(v, dt if k.endswith("conv1.weight") or k.endswith("conv2.weight") else torch.float32)
            for k, v in w.items()}


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("cin,cout", [(64, 32), (128, 64)])
def test_block_16bit_matches_oracle(tb, dtype, cin, cout):
    from trellis_cpp_b200 import ops
    coords, feats, w = _random_case(3000, cin, cout, dtype, cin + cout)
    ref_mask = (feats.astype(np.float64) @ w["to_subdiv.weight"].T.astype(np.float64) + w["to_subdiv.bias"]) > 0
    dt = TORCH_DT[dtype]
    out, child, mask = ops.sparse_c2s(torch.from_numpy(coords).cuda(), _cuda(feats, dt), _params(w, dt), cout,
                                      ext_mask=torch.from_numpy(ref_mask.astype(np.uint8)).cuda(),
                                      out_dtype=torch.float32)
    ops.check_device()
    ref, ref_child, _ = oracle.c2s_block(coords, feats, w, cout, ext_mask=ref_mask.astype(np.uint8))
    assert np.array_equal(child.cpu().numpy(), ref_child)
    assert out.shape == (ref_child.shape[0], cout)
    assert max_rel(out.cpu().numpy(), ref) < 1e-2


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_block_mask_from_logits(tb, dtype):
    from trellis_cpp_b200 import ops
    cin, cout = 64, 32
    coords, feats, w = _random_case(2500, cin, cout, dtype, 77)
    logits = feats.astype(np.float64) @ w["to_subdiv.weight"].T.astype(np.float64) + w["to_subdiv.bias"]
    dt = TORCH_DT[dtype]
    out, child, mask = ops.sparse_c2s(torch.from_numpy(coords).cuda(), _cuda(feats, dt), _params(w, dt), cout,
                                      out_dtype=torch.float32)
    ops.check_device()
    mask = mask.cpu().numpy().astype(bool)
    sure = np.abs(logits) > 1e-4
    assert np.array_equal(mask[sure], (logits > 0)[sure])
    ref, ref_child, _ = oracle.c2s_block(coords, feats, w, cout, ext_mask=mask.astype(np.uint8))
    assert np.array_equal(child.cpu().numpy(), ref_child)
    assert max_rel(out.cpu().numpy(), ref) < (1e-4 if dtype == "f32" else 1e-2)


def test_block_batch_column_and_bf16_output(tb):
    from trellis_cpp_b200 import ops
    cin, cout = 64, 32
    coords, feats, w = _random_case(2000, cin, cout, "bf16", 5)
    coords4 = np.concatenate([np.zeros((coords.shape[0], 1), np.int32), coords], 1)
    mask = (np.random.default_rng(5).random((coords.shape[0], 8)) < 0.4).astype(np.uint8)
    dt = torch.bfloat16
    out, child, _ = ops.sparse_c2s(torch.from_numpy(coords4).cuda(), _cuda(feats, dt), _params(w, dt), cout,
                                   ext_mask=torch.from_numpy(mask).cuda())
    ops.check_device()
    assert out.dtype == torch.bfloat16
    ref, ref_child, _ = oracle.c2s_block(coords, feats, w, cout, ext_mask=mask)
    assert np.array_equal(child.cpu().numpy()[:, 1:], ref_child)
    assert np.all(child.cpu().numpy()[:, 0] == 0)
    assert max_rel(out.float().cpu().numpy(), ref) < 1e-2


def test_empty_mask_gives_no_children(tb):
    from trellis_cpp_b200 import ops
    coords, feats, w = _random_case(500, 64, 32, "bf16", 9)
    dt = torch.bfloat16
    out, child, mask = ops.sparse_c2s(torch.from_numpy(coords).cuda(), _cuda(feats, dt), _params(w, dt), 32,
                                      ext_mask=torch.zeros((500, 8), dtype=torch.uint8, device="cuda"))
    ops.check_device()
    assert out.shape == (0, 32) and child.shape == (0, 3)


def test_too_few_children_reports_count(tb):
    from trellis_cpp_b200 import ops
    coords, feats, w = _random_case(400, 64, 32, "bf16", 13)
    mask = np.ones((400, 8), np.uint8)
    dt = torch.bfloat16
    with pytest.raises(ops.TBError) as e:
        ops.sparse_c2s(torch.from_numpy(coords).cuda(), _cuda(feats, dt), _params(w, dt), 32,
                       ext_mask=torch.from_numpy(mask).cuda(), max_children=1000)
    assert e.value.status == 6            # TB_ERR_TOO_LARGE
    ops.check_device()


def test_unsupported_widths_report_status(tb):
    from trellis_cpp_b200 import ops
    coords, feats, w = _random_case(100, 64, 32, "bf16", 3)
    dt = torch.bfloat16
    w["conv1.weight"] = np.zeros((8 * 36, 27, 64), np.float32)
    w["conv2.weight"] = np.zeros((36, 27, 36), np.float32)
    w["conv1.bias"] = np.zeros(8 * 36, np.float32)
    w["conv2.bias"] = np.zeros(36, np.float32)
    with pytest.raises(ops.TBError) as e:          # cout = 36 is not a multiple of cin / 8 = 8
        ops.sparse_c2s(torch.from_numpy(coords).cuda(), _cuda(feats, dt), _params(w, dt), 36)
    assert e.value.status == 2
