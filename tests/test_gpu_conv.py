"""GPU submanifold conv vs the CPU oracle (fp64 on the exact operands the GPU sees) and vs
the golden outputs of the reference's torch restatement.

Tolerances (max|d| / max|ref|, the reference's metric): 1e-2 for bf16/f16 operands and
1e-4 for fp32 operands, as the path's contract states; with fp32 outputs on identical
operands the only difference is fp32 accumulation order, checked at 1e-4 as well."""
import numpy as np
import pytest
import torch

import oracle
from conftest import max_rel, random_voxels, round_to

pytestmark = pytest.mark.gpu

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}
TOL = {"bf16": 1e-2, "f16": 1e-2, "f32": 1e-4}


def _run(coords, feats, weight, bias, dtype, epi="none", out_dtype=None, nbr=None, path="auto"):
    from trellis_cpp_b200 import ops
    ops.set_conv_path(path)
    dt = TORCH_DT[dtype]
    c = torch.from_numpy(np.ascontiguousarray(coords, dtype=np.int32)).cuda()
    if nbr is None:
        nbr = ops.build_neighbor_table(c)
    f = torch.from_numpy(np.ascontiguousarray(feats, dtype=np.float32)).cuda().to(dt)
    co = weight.shape[0]
    w = torch.from_numpy(np.ascontiguousarray(weight, dtype=np.float32).reshape(co, 27, -1)).cuda().to(dt)
    b = None if bias is None else torch.from_numpy(np.ascontiguousarray(bias, dtype=np.float32)).cuda()
    try:
        out = ops.sparse_submconv(f, nbr, w, b, epi=epi, out_dtype=TORCH_DT[out_dtype] if out_dtype else None)
        ops.check_device()
    finally:
        ops.set_conv_path("auto")
    return out.float().cpu().numpy(), nbr


def _problem(n, ci, co, box, seed, dtype):
    rng = np.random.default_rng(seed)
    coords = random_voxels(n, box, seed)
    feats = round_to(rng.standard_normal((n, ci)).astype(np.float32), dtype)
    w = round_to((rng.standard_normal((co, 27, ci)) / np.sqrt(27 * ci)).astype(np.float32), dtype)
    b = (0.1 * rng.standard_normal(co)).astype(np.float32)
    return coords, feats, w, b


def test_golden_fp32_mode(tb, golden):
    g = golden["submconv"]
    out, _ = _run(g["coords"], g["feats"], g["weight"], g["bias"], "f32")
    assert max_rel(out, g["conv_out"]) < 1e-4


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_golden_half_modes(tb, golden, dtype):
    g = golden["submconv"]
    fr = round_to(g["feats"], dtype)
    out, nbr = _run(g["coords"], fr, g["weight"], g["bias"], dtype, out_dtype="f32")
    # against the reference's own fp32 output (operand rounding included) ...
    assert max_rel(out, g["conv_out"]) < TOL[dtype]
    # ... and against the oracle on the identical rounded operands
    ref = oracle.submconv(nbr.cpu().numpy(), fr, g["weight"], g["bias"])
    assert max_rel(out, ref) < 1e-4


SHAPES = [(16, 16), (32, 32), (64, 64), (64, 128), (128, 64), (128, 128), (256, 256), (32, 128), (256, 32),
          (64, 512), (512, 512), (64, 16), (192, 48), (64, 32), (32, 64)]


@pytest.mark.parametrize("path", ["gather", "brick", "pair"])
@pytest.mark.parametrize("ci,co", SHAPES)
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_channel_shapes(tb, ci, co, dtype, path):
    if path == "brick" and ci % 64:
        pytest.skip("the brick kernel takes ci multiples of 64")
    if path == "pair" and not (ci in (32, 64) and co in (32, 64)):
        pytest.skip("the pair kernel takes ci and co in {32, 64}")
    coords, feats, w, b = _problem(3000, ci, co, 20, ci * 7 + co, dtype)
    out, nbr = _run(coords, feats, w, b, dtype, out_dtype="f32", path=path)
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, b)
    assert max_rel(out, ref) < 1e-4


@pytest.mark.parametrize("ci,co", [(64, 64), (24, 40), (3, 5)])
def test_fp32_mode_shapes(tb, ci, co):
    coords, feats, w, b = _problem(2000, ci, co, 18, ci + co, "f32")
    out, nbr = _run(coords, feats, w, b, "f32")
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, b)
    assert max_rel(out, ref) < 1e-4


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
def test_silu_epilogue_and_low_precision_output(tb, dtype):
    coords, feats, w, b = _problem(2500, 64, 64, 18, 3, dtype)
    out, nbr = _run(coords, feats, w, b, dtype, epi="silu")
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, b, silu=True)
    assert max_rel(out, ref) < TOL[dtype]


@pytest.mark.parametrize("path,ci", [("gather", 64), ("brick", 64), ("pair", 64), ("pair", 32)])
@pytest.mark.parametrize("n", [1, 2, 127, 128, 129, 255, 256, 257, 1000])
def test_sizes_and_partial_tiles(tb, n, path, ci):
    coords, feats, w, b = _problem(n, ci, 64, 16, n, "bf16")
    out, nbr = _run(coords, feats, w, b, "bf16", out_dtype="f32", path=path)
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, b)
    assert max_rel(out, ref) < 1e-4


# Output column blocks of 128 or more run the brick kernel on CTA pairs (two tiles per cluster,
# each CTA streaming half of every weight slice): odd and even tile counts, partial tiles, and
# Co above 256 (several column blocks).
@pytest.mark.parametrize("ci,co", [(64, 128), (128, 256), (256, 512)])
@pytest.mark.parametrize("n", [1, 127, 128, 129, 255, 256, 257, 383, 385, 1000])
def test_brick_pair_sizes_and_partial_tiles(tb, n, ci, co):
    coords, feats, w, b = _problem(n, ci, co, 16, n + co, "bf16")
    out, nbr = _run(coords, feats, w, b, "bf16", out_dtype="f32", path="brick")
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, b)
    assert max_rel(out, ref) < 1e-4


@pytest.mark.parametrize("ci,co", [(128, 128), (256, 256), (64, 512)])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_brick_pair_silu_16bit_output(tb, ci, co, dtype):
    """The pair brick's epilogue: bias, SiLU and a 16-bit output of the operand type."""
    coords, feats, w, b = _problem(2100, ci, co, 18, ci + co + 1, dtype)
    out, nbr = _run(coords, feats, w, b, dtype, epi="silu", path="brick")
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, b, silu=True)
    assert max_rel(out, ref) < TOL[dtype]


@pytest.mark.parametrize("ci", [64, 32])
@pytest.mark.parametrize("misaligned", [False, True])
@pytest.mark.parametrize("n", [1003, 2050, 4097, 6144])
def test_pair_index_fetch_alignment(tb, n, misaligned, ci):
    # the pair kernel copies each tap's tile indices from the 16-byte boundary at or below
    # t * n + r0 (n % 4 selects the offset), and copies them element by element for the last
    # tiles or when the map itself is not 16-byte aligned (a view one int into a buffer)
    from trellis_cpp_b200 import ops
    coords, feats, w, b = _problem(n, ci, 64, 24, n + 7, "bf16")
    c = torch.from_numpy(np.ascontiguousarray(coords, dtype=np.int32)).cuda()
    nbr = ops.build_neighbor_table(c)
    if misaligned:
        holder = torch.empty(27 * n + 1, dtype=torch.int32, device="cuda")
        holder[1:] = nbr
        nbr = holder[1:]
        assert nbr.data_ptr() % 16 != 0
    out, _ = _run(coords, feats, w, b, "bf16", out_dtype="f32", nbr=nbr, path="pair")
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, b)
    assert max_rel(out, ref) < 1e-4


def test_isolated_voxels_only_centre_tap(tb):
    # voxels 2 apart: every row has only its centre tap (t=13)
    g = np.stack(np.meshgrid(*[np.arange(0, 40, 2)] * 3, indexing="ij"), -1).reshape(-1, 3).astype(np.int32)
    rng = np.random.default_rng(1)
    feats = round_to(rng.standard_normal((g.shape[0], 64)).astype(np.float32), "bf16")
    w = round_to(rng.standard_normal((64, 27, 64)).astype(np.float32) / 40, "bf16")
    out, _ = _run(g, feats, w, None, "bf16", out_dtype="f32")
    ref = feats.astype(np.float64) @ w[:, 13, :].T.astype(np.float64)
    assert max_rel(out, ref) < 1e-4


@pytest.mark.parametrize("ci", [32, 64])
def test_duplicate_coordinates(tb, ci):
    rng = np.random.default_rng(2)
    c = rng.integers(0, 9, size=(1500, 3)).astype(np.int32)
    feats = round_to(rng.standard_normal((1500, ci)).astype(np.float32), "bf16")
    w = round_to(rng.standard_normal((32, 27, ci)).astype(np.float32) / 30, "bf16")
    out, nbr = _run(c, feats, w, None, "bf16", out_dtype="f32")
    ref = oracle.submconv(nbr.cpu().numpy(), feats, w, None)
    assert max_rel(out, ref) < 1e-4


def test_deterministic(tb):
    coords, feats, w, b = _problem(5000, 64, 64, 24, 9, "bf16")
    a, nbr = _run(coords, feats, w, b, "bf16")
    c, _ = _run(coords, feats, w, b, "bf16", nbr=nbr)
    assert np.array_equal(a, c)


def test_scattered_voxels_overflow_brick(tb):
    # voxels spread over a large grid in random order: tile neighbor ranges exceed the brick
    # capacity, so rows come through the global-memory fallback
    rng = np.random.default_rng(5)
    coords = random_voxels(6000, 200, 5)
    rng.shuffle(coords)
    feats = round_to(rng.standard_normal((6000, 64)).astype(np.float32), "bf16")
    w = round_to((rng.standard_normal((64, 27, 64)) / 40).astype(np.float32), "bf16")
    for path in ("brick", "pair"):
        out, nbr = _run(coords, feats, w, None, "bf16", out_dtype="f32", path=path)
        ref = oracle.submconv(nbr.cpu().numpy(), feats, w, None)
        assert max_rel(out, ref) < 1e-4, path


def test_unsupported_shape_reports_status(tb):
    from trellis_cpp_b200 import ops
    coords, feats, w, b = _problem(300, 48, 64, 10, 1, "bf16")
    with pytest.raises(ops.TBError) as e:
        _run(coords, feats, w, b, "bf16")
    assert e.value.status == 2


def _sample_rows(n, k, seed):
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([np.arange(min(n, 256)), np.arange(max(0, n - 256), n),
                                     rng.integers(0, n, k)]))
    return rows


@pytest.mark.parametrize("name,ci,co,dtype,path", [("c2", 256, 256, "f16", "auto"), ("c4", 64, 64, "bf16", "auto"),
                                                   ("c4", 64, 64, "bf16", "gather"), ("c4", 64, 64, "bf16", "brick"),
                                                   ("c4", 64, 64, "bf16", "pair"),
                                                   ("c5_32", 32, 32, "f16", "auto"), ("c5_512", 512, 512, "f16", "auto")])
def test_config_full_size_sampled_rows(tb, name, ci, co, dtype, path):
    from trellis_cpp_b200 import ops, synth
    ops.set_conv_path(path)
    coords = synth.coords_for(name)
    n = coords.shape[0]
    rng = np.random.default_rng(11)
    dt = TORCH_DT[dtype]
    c = torch.from_numpy(coords).cuda()
    nbr = ops.build_neighbor_table(c)
    g = torch.Generator(device="cuda").manual_seed(5)
    f = torch.randn((n, ci), device="cuda", generator=g).to(dt)
    w = (torch.randn((co, 27, ci), device="cuda", generator=g) / np.sqrt(27 * ci)).to(dt)
    b = (0.01 * torch.randn(co, device="cuda", generator=g)).float()
    try:
        out = ops.sparse_submconv(f, nbr, w, b, out_dtype=torch.float32)
        ops.check_device()
    finally:
        ops.set_conv_path("auto")
    rows = _sample_rows(n, 3000, 3)
    ref = oracle.submconv_rows(nbr.cpu().numpy(), f.float().cpu().numpy(), w.float().cpu().numpy(), rows,
                               b.cpu().numpy())
    assert max_rel(out[torch.from_numpy(rows).cuda()].cpu().numpy(), ref) < 1e-4
    del rng


def test_c4_two_stacked_convs(tb):
    # the benchmark workload: conv -> SiLU -> conv at C=64 bf16 on the res-1024 shell
    from trellis_cpp_b200 import ops, synth
    coords = synth.coords_for("c4")
    n = coords.shape[0]
    c = torch.from_numpy(coords).cuda()
    nbr = ops.build_neighbor_table(c)
    g = torch.Generator(device="cuda").manual_seed(6)
    f = torch.randn((n, 64), device="cuda", generator=g).bfloat16()
    w1 = (torch.randn((64, 27, 64), device="cuda", generator=g) / np.sqrt(27 * 64)).bfloat16()
    w2 = (torch.randn((64, 27, 64), device="cuda", generator=g) / np.sqrt(27 * 64)).bfloat16()
    h = ops.sparse_submconv(f, nbr, w1, None, epi="silu")
    o = ops.sparse_submconv(h, nbr, w2, None, out_dtype=torch.float32)
    ops.check_device()
    rows = _sample_rows(n, 2000, 4)
    nb = nbr.cpu().numpy()
    # conv 2 checked on the exact bf16 intermediate the GPU produced
    ref2 = oracle.submconv_rows(nb, h.float().cpu().numpy(), w2.float().cpu().numpy(), rows)
    assert max_rel(o[torch.from_numpy(rows).cuda()].cpu().numpy(), ref2) < 1e-4
    # conv 1 (with SiLU, bf16 output) on the same rows
    ref1 = oracle.submconv_rows(nb, f.float().cpu().numpy(), w1.float().cpu().numpy(), rows, silu=True)
    assert max_rel(h[torch.from_numpy(rows).cuda()].float().cpu().numpy(), ref1) < 1e-2


def test_c1_full_config_fp32_every_row(tb):
    """Configuration C1 at its own size: the res-64 band (12,660 voxels), Cin = Cout = 64, fp32
    operands (the reference's --f32 precision mode, src/sparse.cpp:16-19), features N(0,1),
    weights N(0, 1/(27*64)), bias 0. Every output row against the oracle at 1e-4."""
    from trellis_cpp_b200 import ops, synth
    coords = synth.coords_for("c1")
    n = coords.shape[0]
    assert n == 12660
    rng = np.random.default_rng(101)
    feats = rng.standard_normal((n, 64)).astype(np.float32)
    w = (rng.standard_normal((64, 27, 64)) / np.sqrt(27 * 64)).astype(np.float32)
    out, nbr = _run(coords, feats, w, np.zeros(64, np.float32), "f32")
    nb = nbr.cpu().numpy()
    assert np.array_equal(nb, oracle.build_neighbor_table(coords))
    ref = oracle.submconv(nb, feats, w, np.zeros(64, np.float32))
    assert out.shape == ref.shape
    assert max_rel(out, ref) < 1e-4
