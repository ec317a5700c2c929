"""GGUF checkpoints and the hr_slat.bin dump, read through the C ABI without a GPU.

The GGUF files are written by gguf-py's GGUFWriter, the writer the reference's tools/convert.py
uses (conv weights [Co,27,Ci] as F16, 1-D parameters as F32, the config JSON as
`trellis.config_json`); the reader must return the same names, shapes, types, strings and
bytes. The slat file follows src/decode_replay.cpp:19-28."""
import json

import numpy as np
import pytest

gguf = pytest.importorskip("gguf")


def _write_model(path, alignment=None, extra=True):
    rng = np.random.default_rng(0)
    t = {
        "blocks.0.conv.weight": rng.standard_normal((16, 27, 8)).astype(np.float16),   # [Co,27,Ci]
        "blocks.0.conv.bias": rng.standard_normal(16).astype(np.float32),
        "blocks.0.mlp.0.weight": rng.standard_normal((64, 16)).astype(np.float16),
        "blocks.0.norm.weight": rng.standard_normal(16).astype(np.float32),
        "up.to_subdiv.weight": rng.standard_normal((8, 16)).astype(np.float32),
    }
    w = gguf.GGUFWriter(str(path), "trellis2-shape-dec")
    if alignment:
        w.add_custom_alignment(alignment)
    w.add_string("trellis.config_json", json.dumps({"channels": [16, 8]}))
    w.add_string("general.name", "shape_dec")
    if extra:
        w.add_array("test.int_array", [1, 2, 3])
        w.add_array("test.str_array", ["a", "bc"])
        w.add_uint32("test.u32", 7)
        w.add_float32("test.f32", 0.5)
        w.add_bool("test.bool", True)
    for name, a in t.items():
        w.add_tensor(name, a)
    bf = (rng.standard_normal((4, 6)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    w.add_tensor("raw.bf16", bf, raw_dtype=gguf.GGMLQuantizationType.BF16)
    t["raw.bf16"] = bf
    q = np.zeros((2, 34), dtype=np.uint8)      # two Q8_0 blocks of 32 values: listed, not readable
    w.add_tensor("raw.q8", q, raw_dtype=gguf.GGMLQuantizationType.Q8_0)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return t


@pytest.mark.parametrize("alignment", [None, 64])
def test_gguf_round_trip(tb, tmp_path, alignment):
    from trellis_cpp_b200 import ops
    path = tmp_path / "m.gguf"
    t = _write_model(path, alignment)
    f = ops.GgufFile(path)
    assert f.string("general.architecture") == "trellis2-shape-dec"
    assert json.loads(f.string("trellis.config_json")) == {"channels": [16, 8]}
    assert f.string("no.such.key") is None
    assert set(f.tensors) == set(t) | {"raw.q8"}
    for name, a in t.items():
        _, typ, shape, nbytes = f.tensors[name]
        assert shape == a.shape, name
        assert typ == {np.float16: ops.GGUF_F16, np.float32: ops.GGUF_F32, np.uint16: ops.GGUF_BF16}[a.dtype.type]
        assert nbytes == a.nbytes
        got = f.numpy(name)
        assert got.dtype == a.dtype and np.array_equal(got, a), name
    # the conv weight's bytes are the [Co][27][Ci] layout the conv kernels take
    assert f.numpy("blocks.0.conv.weight").shape == (16, 27, 8)
    _, typ, shape, nbytes = f.tensors["raw.q8"]
    assert typ == 8 and nbytes == 0
    with pytest.raises(ops.TBError):
        f.numpy("raw.q8")
    f.close()


def test_gguf_rejects_bad_files(tb, tmp_path):
    from trellis_cpp_b200 import ops
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOTAGGUF" + bytes(64))
    with pytest.raises(ops.TBError) as e:
        ops.GgufFile(bad)
    assert "not a GGUF" in str(e.value)
    good = tmp_path / "m.gguf"
    _write_model(good, extra=False)
    data = good.read_bytes()
    for cut in (6, 40, len(data) - 160):     # the last cut truncates readable tensor data
        part = tmp_path / f"cut{cut}.gguf"
        part.write_bytes(data[:cut])
        with pytest.raises(ops.TBError):
            ops.GgufFile(part)
    with pytest.raises(ops.TBError):
        ops.GgufFile(tmp_path / "missing.gguf")


def _gguf_one_tensor(ne, ggml_type=0, offset=0, data=b""):
    """A minimal GGUF v3 file: no metadata, one tensor info with the given dims, type and
    offset, 32-byte alignment, then `data`."""
    import struct
    name = b"t"
    head = b"GGUF" + struct.pack("<IQQ", 3, 1, 0)
    info = struct.pack("<Q", len(name)) + name + struct.pack("<I", len(ne))
    info += b"".join(struct.pack("<Q", e) for e in ne) + struct.pack("<IQ", ggml_type, offset)
    body = head + info
    body += bytes((-len(body)) % 32)
    return body + data


@pytest.mark.parametrize("ne,offset", [
    ((1 << 40, 1 << 40, 1 << 40, 1 << 40), 0),   # the element count wraps 2^64 several times
    ((1 << 32, 1 << 32), 0),                     # exactly 2^64 elements: wraps to 0
    ((1 << 31, 1 << 31, 4), 0),                  # 2^64 elements again, over three dims
    ((1 << 30, 1 << 30), 0),                     # no wrap, but 2^62 bytes: past the end
    ((4,), (1 << 64) - 8),                       # the data offset wraps the end-of-file check
])
def test_gguf_rejects_overflowing_tensor_infos(tb, tmp_path, ne, offset):
    from trellis_cpp_b200 import ops
    p = tmp_path / "big.gguf"
    p.write_bytes(_gguf_one_tensor(ne, 0, offset, bytes(64)))
    with pytest.raises(ops.TBError):
        ops.GgufFile(p)


def test_gguf_hand_written_file_parses(tb, tmp_path):
    """The crafted layout itself is valid: four F32 values at offset 0 read back."""
    from trellis_cpp_b200 import ops
    vals = np.arange(4, dtype=np.float32)
    p = tmp_path / "small.gguf"
    p.write_bytes(_gguf_one_tensor((4,), 0, 0, vals.tobytes()))
    f = ops.GgufFile(p)
    np.testing.assert_array_equal(f.numpy("t"), vals)
    f.close()


def test_slat_dump(tb, tmp_path):
    from trellis_cpp_b200 import ops
    rng = np.random.default_rng(2)
    n, res = 500, 64
    coords = rng.integers(0, res, (n, 3)).astype(np.int32)
    feats = rng.standard_normal((n, 32)).astype(np.float32)
    p = tmp_path / "hr_slat.bin"
    with open(p, "wb") as f:
        f.write(np.array([n, res], dtype=np.int32).tobytes())
        f.write(coords.tobytes())
        f.write(feats.tobytes())
    c, x, r = ops.read_slat(p)
    assert r == res and np.array_equal(c, coords) and np.array_equal(x, feats)
    p.write_bytes(p.read_bytes()[:-4])
    with pytest.raises(ops.TBError) as e:
        ops.read_slat(p)
    assert "size does not match" in str(e.value)


@pytest.mark.parametrize("header,tail", [((-1, 64), 0), ((2 ** 31 - 1, 64), 100), ((0x10000000, 64), 64), ((7,), 0)])
def test_slat_rejects_bad_headers(tb, tmp_path, header, tail):
    # a negative count, counts whose data the file cannot hold (including one whose byte size
    # overflows 32 bits), and a header cut short: all rejected before any allocation of N rows
    from trellis_cpp_b200 import ops
    p = tmp_path / "bad.bin"
    p.write_bytes(np.array(header, dtype=np.int32).tobytes() + bytes(tail))
    with pytest.raises(ops.TBError):
        ops.read_slat(p)


def test_slat_empty_dump(tb, tmp_path):
    # N = 0 is a valid (empty) dump; the resolution is passed through as the reference reads it
    from trellis_cpp_b200 import ops
    p = tmp_path / "empty.bin"
    p.write_bytes(np.array([0, 64], dtype=np.int32).tobytes())
    c, x, r = ops.read_slat(p)
    assert c.shape == (0, 3) and x.shape == (0, 32) and r == 64
