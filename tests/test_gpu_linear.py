"""Per-voxel dense layers (tb_linear, tb_layer_norm) vs fp64 references on the exact operands.

Tolerances (max|d| / max|ref|): 1e-4 with fp32 outputs (fp32 accumulation over K <= 4096),
1e-2 with 16-bit outputs (one bf16 rounding of the result), 1e-5 for the fp32 mode and the
LayerNorm with fp32 output."""
import numpy as np
import pytest
import torch

from conftest import max_rel

pytestmark = pytest.mark.gpu


def _silu(x):
    return x / (1.0 + np.exp(-x))


@pytest.mark.parametrize("m,k,n", [(1, 64, 16), (130, 32, 1024), (5000, 64, 7), (300, 16, 100), (257, 128, 300),
                                   (1000, 1024, 4096), (777, 4096, 1024)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_linear_shapes(tb, m, k, n, dtype):
    from trellis_cpp_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    a = torch.randn((m, k), device="cuda", generator=g).to(dtype)
    w = (torch.randn((n, k), device="cuda", generator=g) / np.sqrt(k)).to(dtype)
    b = 0.1 * torch.randn(n, device="cuda", generator=g)
    out = ops.linear(a, w, b, out_dtype=torch.float32)
    ops.check_device()
    ref = a.double().cpu().numpy() @ w.double().cpu().numpy().T + b.double().cpu().numpy()
    assert max_rel(out.cpu().numpy(), ref) < 1e-4


# K a multiple of 64 with 256-column tiles and more than one row block runs on CTA pairs (two row
# blocks per cluster, each CTA loading half of the tile's weight rows): odd and even row-block
# counts, a partial last N tile, the decoder's MLP shapes.
@pytest.mark.parametrize("m,k,n", [(129, 64, 256), (255, 128, 512), (256, 64, 272), (383, 512, 2048), (384, 256, 260),
                                   (14211, 512, 2048), (3968, 4096, 1024)])
def test_linear_pair_shapes(tb, m, k, n):
    from trellis_cpp_b200 import ops
    g = torch.Generator(device="cuda").manual_seed(m * 3 + k + n)
    a = torch.randn((m, k), device="cuda", generator=g).bfloat16()
    w = (torch.randn((n, k), device="cuda", generator=g) / np.sqrt(k)).bfloat16()
    b = 0.1 * torch.randn(n, device="cuda", generator=g)
    r = torch.randn((m, n), device="cuda", generator=g)
    out = ops.linear(a, w, b, act="silu", residual=r, out_dtype=torch.float32)
    ops.check_device()
    ref = _silu(a.double().cpu().numpy() @ w.double().cpu().numpy().T + b.double().cpu().numpy()) \
        + r.double().cpu().numpy()
    assert max_rel(out.cpu().numpy(), ref) < 1e-4


@pytest.mark.parametrize("res_dtype", [torch.float32, torch.bfloat16])
def test_linear_silu_residual_16bit_out(tb, res_dtype):
    from trellis_cpp_b200 import ops
    m, k, n = 2000, 256, 64
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn((m, k), device="cuda", generator=g).bfloat16()
    w = (torch.randn((n, k), device="cuda", generator=g) / np.sqrt(k)).bfloat16()
    b = 0.1 * torch.randn(n, device="cuda", generator=g)
    r = torch.randn((m, n), device="cuda", generator=g).to(res_dtype)
    out = ops.linear(a, w, b, act="silu", residual=r)
    ops.check_device()
    assert out.dtype == torch.bfloat16
    ref = _silu(a.double().cpu().numpy() @ w.double().cpu().numpy().T + b.double().cpu().numpy()) \
        + r.double().cpu().numpy()
    assert max_rel(out.float().cpu().numpy(), ref) < 1e-2
    # in place: the residual buffer is the output
    r2 = r.clone().to(torch.bfloat16)
    ops.linear(a, w, b, act="silu", residual=r2, out=r2)
    ops.check_device()
    assert max_rel(r2.float().cpu().numpy(), _silu(a.double().cpu().numpy() @ w.double().cpu().numpy().T
                                                   + b.double().cpu().numpy()) + r.bfloat16().double().cpu().numpy()) < 1e-2


def test_linear_fp32_mode(tb):
    from trellis_cpp_b200 import ops
    m, k, n = 333, 40, 7
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn((m, k), device="cuda", generator=g)
    w = torch.randn((n, k), device="cuda", generator=g)
    b = torch.randn(n, device="cuda", generator=g)
    r = torch.randn((m, n), device="cuda", generator=g)
    out = ops.linear(a, w, b, act="silu", residual=r)
    ops.check_device()
    ref = _silu(a.double().cpu().numpy() @ w.double().cpu().numpy().T + b.double().cpu().numpy()) + r.double().cpu().numpy()
    assert max_rel(out.cpu().numpy(), ref) < 1e-5


def test_linear_unsupported_k(tb):
    from trellis_cpp_b200 import ops
    a = torch.zeros((10, 48), device="cuda", dtype=torch.bfloat16)
    w = torch.zeros((16, 48), device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ops.TBError) as e:
        ops.linear(a, w)
    assert e.value.status == 2


@pytest.mark.parametrize("c,eps,affine,act", [(64, 1e-5, False, "none"), (1024, 1e-6, True, "silu"), (40, 1e-6, True, "none")])
def test_layer_norm(tb, c, eps, affine, act):
    from trellis_cpp_b200 import ops
    n = 3000
    g = torch.Generator(device="cuda").manual_seed(c)
    x = 3 + 2 * torch.randn((n, c), device="cuda", generator=g)
    w = 1 + 0.1 * torch.randn(c, device="cuda", generator=g) if affine else None
    b = 0.1 * torch.randn(c, device="cuda", generator=g) if affine else None
    out = ops.layer_norm(x, w, b, eps=eps, act=act)
    ops.check_device()
    xd = x.double().cpu().numpy()
    y = (xd - xd.mean(1, keepdims=True)) / np.sqrt(xd.var(1, keepdims=True) + eps)
    if affine:
        y = y * w.double().cpu().numpy() + b.double().cpu().numpy()
    if act == "silu":
        y = _silu(y)
    assert max_rel(out.cpu().numpy(), y) < 1e-5
