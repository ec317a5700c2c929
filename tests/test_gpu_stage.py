"""Row-range convs (tb_submconv_range, the reference's submconv_range, src/sparse.cpp:64-79) and
the pipelined host-buffer stage call (tb_submconv_stack_host, the shape of run1,
src/shape_decoder.cpp:34-51).

A conv over row chunks must equal the whole conv: bit for bit for the pair kernel (the benchmark
path) and the fp32 kernel, whose rows are accumulated in the same order whichever CTA computes
them; within 1e-5 relative for the brick and gather kernels, whose two accumulators take taps in
an order that follows the CTA's stage sequence (fp32 rounding differences only). The host call must return exactly what the device path
(map, conv, conv) produces, with one chunk (small N) and with the chunked, overlapped pipeline
(N above two chunks of 131,072 rows)."""
import numpy as np
import pytest
import torch

from conftest import max_rel, random_voxels

pytestmark = pytest.mark.gpu


def _conv_inputs(n, ci, co, dtype, seed, box):
    g = torch.Generator(device="cuda").manual_seed(seed)
    coords = torch.from_numpy(random_voxels(n, box, seed)).cuda()
    f = torch.randn((n, ci), device="cuda", generator=g).to(dtype)
    w = (torch.randn((co, 27, ci), device="cuda", generator=g) / np.sqrt(27 * ci)).to(dtype)
    b = 0.1 * torch.randn(co, device="cuda", generator=g)
    return coords, f, w, b


@pytest.mark.parametrize("ci,co,dtype,path", [(64, 64, torch.bfloat16, "pair"), (128, 64, torch.bfloat16, "brick"),
                                              (64, 256, torch.bfloat16, "brick"),
                                              (32, 32, torch.float16, "gather"), (24, 40, torch.float32, "auto")])
def test_range_chunks_equal_whole_conv(tb, ci, co, dtype, path):
    from trellis_cpp_b200 import ops
    n = 5000
    coords, f, w, b = _conv_inputs(n, ci, co, dtype, ci + co, 30)
    nbr = ops.build_neighbor_table(coords)
    ops.set_conv_path(path)
    try:
        whole = ops.sparse_submconv(f, nbr, w, b, epi="silu", out_dtype=torch.float32)
        parts = torch.full_like(whole, float("nan"))
        for r0, nr in ((0, 1024), (1024, 256), (1280, 2560), (3840, n - 3840)):
            ops.sparse_submconv_range(f, nbr, w, b, r0, nr, parts, epi="silu")
        ops.check_device()
    finally:
        ops.set_conv_path("auto")
    assert not torch.isnan(parts).any()
    if path in ("pair", "auto"):
        assert torch.equal(whole, parts)
    else:
        assert max_rel(parts.cpu().numpy(), whole.cpu().numpy()) < 1e-5


def test_range_writes_only_its_rows(tb):
    from trellis_cpp_b200 import ops
    n = 3000
    coords, f, w, b = _conv_inputs(n, 64, 64, torch.bfloat16, 3, 26)
    nbr = ops.build_neighbor_table(coords)
    whole = ops.sparse_submconv(f, nbr, w, b)
    out = torch.zeros_like(whole)
    ops.sparse_submconv_range(f, nbr, w, b, 512, 1000, out)
    ops.check_device()
    assert torch.equal(out[512:1512], whole[512:1512])
    assert not out[:512].any() and not out[1512:].any()


@pytest.mark.parametrize("ci,co,dtype,path", [(64, 64, torch.bfloat16, "pair"), (128, 64, torch.bfloat16, "brick"),
                                              (128, 128, torch.bfloat16, "brick"),
                                              (32, 32, torch.float16, "gather"), (24, 40, torch.float32, "auto")])
def test_range_any_start_row(tb, ci, co, dtype, path):
    """Ranges may start and end anywhere: the kernels run the whole tiles that hold the range and
    store only its rows (the slab-local convs of the multi-GPU path start mid-tile)."""
    from trellis_cpp_b200 import ops
    n = 3000
    coords, f, w, b = _conv_inputs(n, ci, co, dtype, 4, 20)
    nbr = ops.build_neighbor_table(coords)
    ops.set_conv_path(path)
    try:
        whole = ops.sparse_submconv(f, nbr, w, b, out_dtype=torch.float32)
        out = torch.zeros_like(whole)
        for r0, nr in ((100, 200), (300, 1), (301, 1000), (1301, 1699)):
            ops.sparse_submconv_range(f, nbr, w, b, r0, nr, out)
        out2 = torch.zeros_like(whole)
        ops.sparse_submconv_range(f, nbr, w, b, 777, 555, out2)
        ops.check_device()
    finally:
        ops.set_conv_path("auto")
    assert not out[:100].any()
    assert not out2[:777].any() and not out2[777 + 555:].any()
    if path in ("pair", "auto"):
        assert torch.equal(out[100:], whole[100:])
        assert torch.equal(out2[777:1332], whole[777:1332])
    else:
        assert max_rel(out[100:].cpu().numpy(), whole[100:].cpu().numpy()) < 1e-5
        assert max_rel(out2[777:1332].cpu().numpy(), whole[777:1332].cpu().numpy()) < 1e-5


def test_range_rejects_bad_bounds(tb):
    from trellis_cpp_b200 import ops
    coords, f, w, b = _conv_inputs(600, 64, 64, torch.bfloat16, 4, 20)
    nbr = ops.build_neighbor_table(coords)
    out = torch.zeros((600, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ops.TBError) as e:
        ops.sparse_submconv_range(f, nbr, w, b, 512, 200, out)      # past the end
    assert e.value.status == 1
    with pytest.raises(ops.TBError):
        ops.sparse_submconv_range(f, nbr, w, b, -1, 10, out)


def _stack_both_ways(coords_np, ci, co, seed):
    from trellis_cpp_b200 import ops
    n = coords_np.shape[0]
    g = torch.Generator(device="cuda").manual_seed(seed)
    f = torch.randn((n, ci), device="cuda", generator=g).bfloat16()
    w1 = (torch.randn((co, 27, ci), device="cuda", generator=g) / np.sqrt(27 * ci)).bfloat16()
    w2 = (torch.randn((co, 27, co), device="cuda", generator=g) / np.sqrt(27 * co)).bfloat16()
    b1 = 0.1 * torch.randn(co, device="cuda", generator=g)
    nbr = ops.build_neighbor_table(torch.from_numpy(coords_np).cuda())
    h = ops.sparse_submconv(f, nbr, w1, b1, epi="silu")
    dev = ops.sparse_submconv(h, nbr, w2, None, out_dtype=torch.float32)
    feats_h = torch.empty((n, ci), dtype=torch.bfloat16).pin_memory()
    feats_h.copy_(f.cpu())
    out_h = torch.empty((n, co), dtype=torch.float32).pin_memory()
    ops.submconv_stack_host(coords_np, feats_h.view(torch.int16).numpy(), [(w1, b1, "silu"), (w2, None, "none")],
                            torch.bfloat16, torch.float32, out=out_h.numpy())
    ops.check_device()
    return dev.cpu(), out_h, nbr, h


def test_stack_host_single_chunk(tb):
    coords = random_voxels(20000, 50, 8)
    dev, host, _, _ = _stack_both_ways(coords, 64, 64, 8)
    assert torch.equal(dev, host)


def test_stack_host_pipelined_chunks(tb):
    # the c4s shell: 1.22M voxels -> nine overlapped chunks
    from trellis_cpp_b200 import synth
    coords = synth.coords_for("c4s")
    assert coords.shape[0] >= 4 * 131072
    dev, host, _, _ = _stack_both_ways(coords, 64, 64, 9)
    assert torch.equal(dev, host)


def test_stack_host_pipelined_shuffled_rows(tb):
    # rows in random order: every chunk reads inputs from every other chunk, so each conv
    # waits for the whole input; the result is still exact
    from trellis_cpp_b200 import synth
    coords = synth.coords_for("c4s")
    perm = np.random.default_rng(3).permutation(coords.shape[0])
    coords = np.ascontiguousarray(coords[perm])
    dev, host, _, _ = _stack_both_ways(coords, 64, 64, 10)
    assert torch.equal(dev, host)
