"""Per-voxel tensors above 2^31 elements through the conv, as the reference's big-tensor stress
tool drives them (src/test_bigop.cpp:95-120 `submconv`, a dense cube at C = 1024 through
blocks.0.0.conv; :138-152 `submconv4096`, the C2S block's conv1 with Co = 8 * 512 = 4096).

Both cases run the real sparse path on a dense cube of voxels in the reference's x, y, z loop
order and check sampled output rows, always including the last 48 rows (whose element offsets
are beyond 2^31), against the CPU oracle on the same bf16 operands at 1e-4 (fp32 outputs, so
only the accumulation order differs). The oracle runs on a compact copy of the sampled rows'
neighbourhoods, so the host never holds the multi-GB tensors."""
import numpy as np
import pytest
import torch

import oracle
from conftest import max_rel

pytestmark = pytest.mark.gpu


def _dense_cube(n):
    """The first n voxels of an s^3 cube, x outermost (src/test_bigop.cpp:98-102)."""
    s = int(np.cbrt(n)) + 1
    i = np.arange(n, dtype=np.int64)
    return np.stack([i // (s * s), (i // s) % s, i % s], axis=1).astype(np.int32)


def _check_rows(nbr, f, w, b, out, rows):
    """Oracle rows `rows` of the conv, on the sampled rows' neighbour rows only."""
    n = f.shape[0]
    r = torch.from_numpy(rows).cuda()
    nb = nbr.view(27, n)[:, r]                                        # [27][k] global rows
    present = nb < n
    u, inv = torch.unique(nb[present], return_inverse=True)          # needed feature rows
    m = u.numel()
    assert m >= rows.size                                             # the centre tap holds every row
    local = torch.full_like(nb, m)
    local[present] = inv.to(torch.int32)
    nbr_c = torch.full((27, m), m, dtype=torch.int32, device="cuda")  # output rows 0..k-1 are the samples
    nbr_c[:, :rows.size] = local
    ref = oracle.submconv_rows(nbr_c.cpu().numpy().reshape(-1), f[u].float().cpu().numpy(),
                               w.float().cpu().numpy(), np.arange(rows.size), b.cpu().numpy())
    return max_rel(out[r].cpu().numpy(), ref)


@pytest.mark.parametrize("n,ci,co", [(2_200_000, 1024, 1024),     # input and output above 2^31 elements
                                     (600_000, 1024, 4096)])      # the C2S conv1 width, output above 2^31
def test_conv_tensors_above_2_31_elements(tb, n, ci, co):
    from trellis_cpp_b200 import ops
    assert max(n * ci, n * co) > 2 ** 31
    coords = torch.from_numpy(_dense_cube(n)).cuda()
    nbr = ops.build_neighbor_table(coords)
    g = torch.Generator(device="cuda").manual_seed(n + co)
    f = torch.randn((n, ci), device="cuda", generator=g).bfloat16()
    w = (torch.randn((co, 27, ci), device="cuda", generator=g) / np.sqrt(27 * ci)).bfloat16()
    b = (0.01 * torch.randn(co, device="cuda", generator=g)).float()
    out = ops.sparse_submconv(f, nbr, w, b, out_dtype=torch.float32)
    ops.check_device()
    rng = np.random.default_rng(n)
    rows = np.unique(np.concatenate([np.arange(16), np.arange(n - 48, n), rng.integers(0, n, 16)]))
    assert rows.max() * co > 2 ** 31
    assert _check_rows(nbr, f, w, b, out, rows) < 1e-4
