"""GGUF container (no GPU): write / read round trips of metadata and tensor bytes, the model
configuration read back from the metadata (model/config.rs:106-247 restated), and the errors
the reference's reader reports (gguf.rs: bad magic, unsupported version, truncated data).
"""
import struct

import numpy as np
import pytest

import oracle as O
from rust_interference_engine_b200 import GgmlType
from rust_interference_engine_b200 import gguf as G
from rust_interference_engine_b200 import model as M


def _tensors(spec, seed=5):
    rng = O.Rng(seed)
    weight = lambda t, r, c: rng.weight(int(t), r, c)
    vec = lambda n, s: rng.vec(n, s)
    norm = lambda n: (1.0 + 0.1 * rng.vec(n, 1.0)).astype(np.float32)
    return list(M.synthetic_tensors(spec, weight, vec, norm))


def test_metadata_and_tensors_round_trip():
    w = G.GgufWriter()
    V = G.ValueType
    vals = [("a.u8", V.UINT8, 200), ("a.i8", V.INT8, -5), ("a.u16", V.UINT16, 60000), ("a.i16", V.INT16, -300),
            ("a.u32", V.UINT32, 4000000000), ("a.i32", V.INT32, -7), ("a.f32", V.FLOAT32, 1.5),
            ("a.bool", V.BOOL, True), ("a.str", V.STRING, "héllo"), ("a.u64", V.UINT64, 1 << 40),
            ("a.i64", V.INT64, -(1 << 40)), ("a.f64", V.FLOAT64, 0.1),
            ("a.arr", V.ARRAY, (V.STRING, ["x", "yz"]))]
    for k, t, v in vals:
        w.kv(k, t, v)
    rng = O.Rng(3)
    data = {"w.q4k": (GgmlType.Q4_K, 3, 512, rng.weight(int(GgmlType.Q4_K), 3, 512)),
            "w.q6k": (GgmlType.Q6_K, 2, 256, rng.weight(int(GgmlType.Q6_K), 2, 256)),
            "w.f32": (GgmlType.F32, 1, 7, np.arange(7, dtype=np.float32))}
    for name, (t, r, c, d) in data.items():
        w.tensor(name, r, c, int(t), d)
    g = G.GgufFile.from_bytes(w.to_bytes())
    assert g.version == 3 and g.alignment == 32
    for k, t, v in vals:
        got = g.get(k)
        assert got.type == t
        if t == V.ARRAY:
            assert [x.value for x in got.value] == v[1]
        elif t == V.FLOAT32:
            assert got.value == np.float32(v)
        else:
            assert got.value == v
    assert g.get_u64("a.i8") is None and g.get_u64("a.u32") == 4000000000 and g.get_bool("a.bool") is True
    for name, (t, r, c, d) in data.items():
        info = g.tensor(name)
        assert info.type == int(t) and info.n_rows == r and info.row_len == c
        assert (g.data_offset + info.offset) % 32 == 0
        assert np.array_equal(g.tensor_data(info).reshape(-1), np.ascontiguousarray(d).view(np.uint8).reshape(-1))


@pytest.mark.parametrize("arch,wtype", [("llama", GgmlType.Q4_0), ("qwen2", GgmlType.Q8_0), ("qwen3", GgmlType.Q4_K),
                                        ("phi3", GgmlType.Q5_0), ("gemma2", GgmlType.Q6_K),
                                        ("qwen3moe", GgmlType.Q4_K), ("qwen2moe", GgmlType.Q8_0)])
def test_config_from_metadata_matches_the_spec(tmp_path, arch, wtype):
    spec = M.SyntheticSpec.tiny(arch, wtype)
    tensors = _tensors(spec)
    path = tmp_path / f"{arch}.gguf"
    G.spec_writer(spec, tensors).write(path)
    g = G.GgufFile.open(path)
    got, want = G.config_from_gguf(g), spec.config()
    for field, _ in M.ModelConfig._fields_:
        assert getattr(got, field) == getattr(want, field), field
    # every tensor comes back byte for byte, in the file's order
    assert [t.name for t in g.tensors] == [t[0] for t in tensors]
    for info, (name, t, rows, cols, data) in zip(g.tensors, tensors):
        assert (info.type, info.n_rows, info.row_len) == (int(t), rows, cols), name
        assert np.array_equal(g.tensor_data(info).reshape(-1), np.ascontiguousarray(data).view(np.uint8).reshape(-1))


def test_reader_errors():
    good = G.spec_writer(M.SyntheticSpec.tiny("qwen3", GgmlType.Q4_0), []).to_bytes()
    with pytest.raises(G.GgufError, match="magic"):
        G.GgufFile.from_bytes(b"GGUX" + good[4:])
    for v in (1, 4):
        with pytest.raises(G.GgufError, match="version"):
            G.GgufFile.from_bytes(good[:4] + struct.pack("<I", v) + good[8:])
    with pytest.raises(G.GgufError, match="end of file"):
        G.GgufFile.from_bytes(good[:40])
    # a tensor whose data runs past the end of the file
    w = G.GgufWriter().kv("general.architecture", G.ValueType.STRING, "qwen3")
    w.tensor("t", 2, 64, int(GgmlType.F32), np.zeros(128, np.float32))
    with pytest.raises(G.GgufError, match="out of bounds"):
        G.GgufFile.from_bytes(w.to_bytes()[:-16])
    with pytest.raises(G.GgufError, match="architecture"):
        G.config_from_gguf(G.GgufFile.from_bytes(G.GgufWriter().to_bytes()))
    bad = G.GgufWriter().kv("general.architecture", G.ValueType.STRING, "rwkv").to_bytes()
    with pytest.raises(G.GgufError, match="supported"):
        G.config_from_gguf(G.GgufFile.from_bytes(bad))
