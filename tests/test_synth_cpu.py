"""Seeded synthetic generators: deterministic, thread-count independent, expected sizes."""
import numpy as np


def test_c1_size_and_determinism(tb):
    from trellis_cpp_b200 import synth
    a = synth.coords_for("c1", nthreads=1)
    b = synth.coords_for("c1", nthreads=5)
    assert np.array_equal(a, b)
    assert 11000 < a.shape[0] < 14000
    d = np.linalg.norm(a[:, 1:] - 32.0, axis=1)
    assert d.min() >= 22 and d.max() < 24


def test_c2_shell_size_and_order(tb):
    from trellis_cpp_b200 import synth
    c = synth.coords_for("c2")
    assert 200_000 < c.shape[0] < 300_000
    # x-major lexicographic order, unique
    key = (c[:, 1].astype(np.int64) << 20) | (c[:, 2].astype(np.int64) << 10) | c[:, 3]
    assert np.all(np.diff(key) > 0)


def test_c3_mask_keeps_about_half(tb):
    from trellis_cpp_b200 import synth
    c = synth.coords_for("c3")
    m = synth.c3_mask(c)
    assert m.shape == (c.shape[0], 8)
    assert 0.3 < m.mean() < 0.6
