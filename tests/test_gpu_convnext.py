"""GPU ConvNeXt block (sparse_convnext, src/sparse.cpp:101-137) vs the CPU oracle and the
golden output of the reference's torch restatement.

The tail is out = x + W2 . silu(W1 . LN(h) + b1) + b2 (LN over channels, eps 1e-6, affine).
Tolerances (max|d| / max|ref|): 1e-4 in the fp32 mode; for bf16/f16 operands 3e-3 against an
oracle that rounds the normalised row and the SiLU activations to the operand type where the
kernel does (what remains is fp32 vs fp64 arithmetic before those roundings, which now and then
puts a value on the other side of a rounding boundary: one bf16 ulp is 3.9e-3 relative), and
1e-2 against the unrounded fp64 result, the tolerance the path states for 16-bit operands."""
import numpy as np
import pytest
import torch

import oracle
from conftest import max_rel, random_voxels, round_to

pytestmark = pytest.mark.gpu

TORCH_DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _tail_ref(h, x, nw, nb, w1, b1, w2, b2, rnd=None):
    """fp64 tail; with rnd the LN output and the activations are rounded to that type first."""
    y = oracle.layer_norm(h.astype(np.float64), nw, nb)
    if rnd:
        y = round_to(y.astype(np.float32), rnd).astype(np.float64)
    a = oracle.silu(y @ w1.T.astype(np.float64) + b1)
    if rnd:
        a = round_to(a.astype(np.float32), rnd).astype(np.float64)
    return a @ w2.T.astype(np.float64) + b2 + x.astype(np.float64)


def _params(c, dtype, seed):
    rng = np.random.default_rng(seed)
    w1 = round_to((rng.standard_normal((4 * c, c)) / np.sqrt(c)).astype(np.float32), dtype)
    w2 = round_to((rng.standard_normal((c, 4 * c)) / np.sqrt(4 * c)).astype(np.float32), dtype)
    nw = (1 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    nb = (0.1 * rng.standard_normal(c)).astype(np.float32)
    b1 = (0.1 * rng.standard_normal(4 * c)).astype(np.float32)
    b2 = (0.1 * rng.standard_normal(c)).astype(np.float32)
    return w1, w2, nw, nb, b1, b2


def _cuda(a, dt=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda().to(dt)


def _run_tail(h, x, w1, w2, nw, nb, b1, b2, dtype, h_dtype="f32", out_dtype="f32"):
    from trellis_cpp_b200 import ops
    dt = TORCH_DT[dtype]
    out = ops.convnext_tail(_cuda(h, TORCH_DT[h_dtype]), _cuda(x, dt), _cuda(nw), _cuda(nb), _cuda(w1, dt), _cuda(b1),
                            _cuda(w2, dt), _cuda(b2), out_dtype=TORCH_DT[out_dtype])
    ops.check_device()
    return out.float().cpu().numpy()


def test_golden_block_fp32(tb, golden):
    # the reference's whole ConvNeXt block (C = 32) in the fp32 mode
    from trellis_cpp_b200 import ops
    g = golden["submconv"]
    c = g["feats"].shape[1]
    coords = torch.from_numpy(g["coords"]).cuda()
    nbr = ops.build_neighbor_table(coords)
    out = ops.sparse_convnext(_cuda(g["feats"]), nbr, _cuda(g["weight"].reshape(c, 27, c)), _cuda(g["bias"]),
                              _cuda(g["norm.weight"]), _cuda(g["norm.bias"]), _cuda(g["mlp.0.weight"]),
                              _cuda(g["mlp.0.bias"]), _cuda(g["mlp.2.weight"]), _cuda(g["mlp.2.bias"]))
    ops.check_device()
    assert max_rel(out.cpu().numpy(), g["block_out"]) < 1e-4


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("c", [64, 128, 256])
def test_tail_tensor_core(tb, c, dtype):
    rng = np.random.default_rng(c + (dtype == "f16"))
    n = 3000
    h = (0.5 + 2.0 * rng.standard_normal((n, c))).astype(np.float32)
    x = round_to(rng.standard_normal((n, c)).astype(np.float32), dtype)
    w1, w2, nw, nb, b1, b2 = _params(c, dtype, c)
    out = _run_tail(h, x, w1, w2, nw, nb, b1, b2, dtype)
    assert max_rel(out, _tail_ref(h, x, nw, nb, w1, b1, w2, b2, rnd=dtype)) < 3e-3
    assert max_rel(out, _tail_ref(h, x, nw, nb, w1, b1, w2, b2)) < 1e-2


@pytest.mark.parametrize("n", [1, 127, 128, 129, 1000])
def test_tail_partial_tiles(tb, n):
    rng = np.random.default_rng(n)
    c = 64
    h = rng.standard_normal((n, c)).astype(np.float32)
    x = round_to(rng.standard_normal((n, c)).astype(np.float32), "bf16")
    w1, w2, nw, nb, b1, b2 = _params(c, "bf16", 7)
    out = _run_tail(h, x, w1, w2, nw, nb, b1, b2, "bf16")
    assert max_rel(out, _tail_ref(h, x, nw, nb, w1, b1, w2, b2, rnd="bf16")) < 3e-3


def test_tail_16bit_h_and_output(tb):
    rng = np.random.default_rng(5)
    n, c = 2000, 128
    h = round_to(rng.standard_normal((n, c)).astype(np.float32), "bf16")
    x = round_to(rng.standard_normal((n, c)).astype(np.float32), "bf16")
    w1, w2, nw, nb, b1, b2 = _params(c, "bf16", 9)
    out = _run_tail(h, x, w1, w2, nw, nb, b1, b2, "bf16", h_dtype="bf16", out_dtype="bf16")
    assert max_rel(out, _tail_ref(h, x, nw, nb, w1, b1, w2, b2)) < 1e-2


def test_tail_fp32_mode_odd_width(tb):
    rng = np.random.default_rng(11)
    n, c = 700, 40
    h = rng.standard_normal((n, c)).astype(np.float32)
    x = rng.standard_normal((n, c)).astype(np.float32)
    w1, w2, nw, nb, b1, b2 = _params(c, "f32", 11)
    out = _run_tail(h, x, w1, w2, nw, nb, b1, b2, "f32")
    assert max_rel(out, _tail_ref(h, x, nw, nb, w1, b1, w2, b2)) < 1e-4


def test_block_bf16_matches_oracle(tb):
    # conv (pair kernel at C = 64) then the tensor-core tail, against the fp64 oracle
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(21)
    n, c = 6000, 64
    coords = random_voxels(n, 28, 21)
    feats = round_to(rng.standard_normal((n, c)).astype(np.float32), "bf16")
    cw = round_to((rng.standard_normal((c, 27, c)) / np.sqrt(27 * c)).astype(np.float32), "bf16")
    cb = (0.1 * rng.standard_normal(c)).astype(np.float32)
    w1, w2, nw, nb, b1, b2 = _params(c, "bf16", 21)
    nbr = ops.build_neighbor_table(torch.from_numpy(coords).cuda())
    dt = torch.bfloat16
    out = ops.sparse_convnext(_cuda(feats, dt), nbr, _cuda(cw, dt), _cuda(cb), _cuda(nw), _cuda(nb), _cuda(w1, dt),
                              _cuda(b1), _cuda(w2, dt), _cuda(b2), out_dtype=torch.float32)
    ops.check_device()
    h = oracle.submconv(nbr.cpu().numpy(), feats, cw, cb)
    assert max_rel(out.cpu().numpy(), _tail_ref(h, feats, nw, nb, w1, b1, w2, b2)) < 1e-2


@pytest.mark.parametrize("c", [32, 512, 1024])
def test_tail_wide_and_narrow_widths(tb, c):
    # widths outside the fused kernel: LayerNorm, mlp.0 + SiLU and mlp.2 + residual as passes
    rng = np.random.default_rng(c)
    n = 700
    h = (0.5 + 2.0 * rng.standard_normal((n, c))).astype(np.float32)
    x = round_to(rng.standard_normal((n, c)).astype(np.float32), "bf16")
    w1, w2, nw, nb, b1, b2 = _params(c, "bf16", c)
    out = _run_tail(h, x, w1, w2, nw, nb, b1, b2, "bf16")
    assert max_rel(out, _tail_ref(h, x, nw, nb, w1, b1, w2, b2, rnd="bf16")) < 3e-3
    assert max_rel(out, _tail_ref(h, x, nw, nb, w1, b1, w2, b2)) < 1e-2


def test_unsupported_width_reports_status(tb):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(1)
    n, c = 100, 80          # neither a fused width, 16, 32 nor a multiple of 64
    w1, w2, nw, nb, b1, b2 = _params(c, "bf16", 1)
    with pytest.raises(ops.TBError) as e:
        _run_tail(rng.standard_normal((n, c)).astype(np.float32), np.zeros((n, c), np.float32),
                  w1, w2, nw, nb, b1, b2, "bf16")
    assert e.value.status == 2
