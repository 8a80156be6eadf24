"""GGUF container tests, restating laya-rust ``tests/gguf.rs`` for the Python
writer/reader the random-init generator uses, plus the loader validations of
``gguf.rs:289-357`` exercised through the C oracle."""
import os
import struct

import numpy as np
import pytest

from laya_rust_b200 import gguf
from laya_rust_b200.gguf import Value


def test_metadata_value_types_round_trip(tmp_path):
    """tests/gguf.rs:14-120"""
    path = str(tmp_path / "kv.gguf")
    w = gguf.Writer()
    w.add_kv("general.architecture", Value(gguf.STR, "laya"))
    w.add_kv("laya.u8", Value(gguf.U8, 200))
    w.add_kv("laya.i8", Value(gguf.I8, -100))
    w.add_kv("laya.u16", Value(gguf.U16, 60000))
    w.add_kv("laya.i16", Value(gguf.I16, -30000))
    w.add_kv("laya.u32", Value(gguf.U32, 4_000_000_000))
    w.add_kv("laya.i32", Value(gguf.I32, -2_000_000_000))
    w.add_kv("laya.f32", Value(gguf.F32, 0.35355338))
    w.add_kv("laya.bool_t", Value(gguf.BOOL, True))
    w.add_kv("laya.bool_f", Value(gguf.BOOL, False))
    w.add_kv("laya.u64", Value(gguf.U64, 2 ** 64 - 1))
    w.add_kv("laya.i64", Value(gguf.I64, -2 ** 63))
    w.add_kv("laya.f64", Value(gguf.F64, 1.0e-5))
    w.add_kv("laya.str", Value(gguf.STR, "现代BERT · [MASK] 50284"))
    w.add_kv("laya.arr_i32", Value(gguf.ARR, [Value(gguf.I32, i) for i in (1, 2, 3)]))
    w.add_kv("laya.arr_f32", Value(gguf.ARR, [Value(gguf.F32, 1.5), Value(gguf.F32, -2.25)]))
    w.add_kv("laya.arr_str", Value(gguf.ARR, [Value(gguf.STR, "a b"), Value(gguf.STR, "c d")]))
    w.add_kv("laya.arr_nested", Value(gguf.ARR, [
        Value(gguf.ARR, [Value(gguf.U8, 1), Value(gguf.U8, 2)]),
        Value(gguf.ARR, [Value(gguf.U8, 3)])]))
    w.add_tensor("t.f32", [3, 4], gguf.T_F32, gguf.f32_bytes(np.arange(12) * 0.5))
    w.add_tensor("t.f16", [8], gguf.T_F16,
                 gguf.f16_bytes([0.0, 1.0, -1.0, 0.5, 0.25, 1e-5, 1234.0, -0.0]))
    w.add_tensor("t.oneelem", [1], gguf.T_F32, gguf.f32_bytes([42.0]))
    w.write(path)

    h = gguf.read(path)
    assert h.data_off % gguf.ALIGNMENT == 0
    for t in h.tensors:
        assert t.offset % gguf.ALIGNMENT == 0
    assert h.str_or("general.architecture", "?") == "laya"
    assert h.u64_or("laya.u8", 0) == 200
    assert h.u64_or("laya.u32", 0) == 4_000_000_000
    assert h.u64_or("laya.u64", 0) == 2 ** 64 - 1
    assert h.f32_or("laya.f32", 0.0) == float(np.float32(0.35355338))
    assert h.f32_or("laya.f64", 0.0) == float(np.float32(1.0e-5))
    assert h.get("laya.bool_t").v is True and h.get("laya.bool_f").v is False
    assert h.get("laya.str").as_str() == "现代BERT · [MASK] 50284"
    assert h.get("laya.arr_i32").as_f32s() == [], "int arrays are not float arrays"
    assert h.get("laya.arr_str").as_strs() == ["a b", "c d"]
    assert h.get("laya.arr_f32").as_f32s() == [1.5, -2.25]
    outer = h.get("laya.arr_nested")
    assert outer.ty == gguf.ARR and len(outer.v) == 2 and len(outer.v[0].v) == 2
    assert h.get("laya.i64").as_u64() == (-2 ** 63) & 0xFFFFFFFFFFFFFFFF
    t32 = h.tensor("t.f32")
    assert t32.dims == [3, 4] and t32.ty == gguf.T_F32 and t32.nbytes() == 48
    assert np.array_equal(h.f32("t.f32").ravel(), np.arange(12, dtype=np.float32) * 0.5)
    t16 = h.tensor("t.f16")
    assert t16.nbytes() == 16
    back = h.f32("t.f16").ravel()
    assert back[1] == 1.0 and back[6] == 1234.0 and back[7] == 0.0


def test_key_rules():
    """tests/gguf.rs:172-184"""
    for k in ["laya.temperature.0", "general.architecture", "laya.rope_theta.full",
              "tokenizer.ggml.mask_token_id"]:
        assert gguf.key_ok(k)
    for k in ["Laya.temperature", "laya.temperature-by-options", "laya.temperature:2",
              "laya..temperature", ".laya", ""]:
        assert not gguf.key_ok(k)


def test_tensor_count_and_types(tmp_path):
    """tests/gguf.rs:186-210"""
    path = str(tmp_path / "count.gguf")
    w = gguf.Writer()
    w.add_kv("general.architecture", Value(gguf.STR, "laya"))
    w.add_tensor("a", [1024], gguf.T_F32, gguf.f32_bytes(np.ones(1024)))
    w.add_tensor("b", [3072, 1024], gguf.T_F16, gguf.f16_bytes(np.full(3072 * 1024, 0.5)))
    w.write(path)
    h = gguf.read(path)
    assert len(h.tensors) == 2
    b = h.tensor("b")
    assert b.dims == [3072, 1024] and b.nbytes() == 3072 * 1024 * 2
    assert h.tensor("a").offset == 0
    assert h.tensor("b").offset == 4096


def test_writer_rejects_bad_input():
    """gguf.rs:390-426: illegal keys, names, dims, sizes and duplicates."""
    w = gguf.Writer()
    with pytest.raises(gguf.GGUFError):
        w.add_kv("Bad.Key", Value(gguf.U8, 1))
    with pytest.raises(gguf.GGUFError):
        w.add_tensor("x" * 65, [1], gguf.T_F32, b"\0" * 4)
    with pytest.raises(gguf.GGUFError):
        w.add_tensor("t", [1, 1, 1, 1, 1], gguf.T_F32, b"\0" * 4)
    with pytest.raises(gguf.GGUFError):
        w.add_tensor("t", [2], gguf.T_F32, b"\0" * 4)
    w.add_tensor("t", [1], gguf.T_F32, b"\0" * 4)
    with pytest.raises(gguf.GGUFError):
        w.add_tensor("t", [1], gguf.T_F32, b"\0" * 4)


def _write_small(path):
    w = gguf.Writer()
    w.add_kv("general.architecture", Value(gguf.STR, "laya"))
    w.add_tensor("a", [8], gguf.T_F32, gguf.f32_bytes(np.ones(8)))
    w.write(path)


def test_reader_validation(tmp_path):
    """gguf.rs:289-357: magic, version, truncation, misaligned offsets."""
    p = str(tmp_path / "ok.gguf")
    _write_small(p)
    raw = open(p, "rb").read()
    bad = str(tmp_path / "bad.gguf")
    open(bad, "wb").write(b"XXXX" + raw[4:])
    with pytest.raises(gguf.GGUFError, match="not a GGUF"):
        gguf.read(bad)
    open(bad, "wb").write(raw[:4] + struct.pack("<I", 2) + raw[8:])
    with pytest.raises(gguf.GGUFError, match="version"):
        gguf.read(bad)
    open(bad, "wb").write(raw[:-8])
    with pytest.raises(gguf.GGUFError, match="outside the file"):
        gguf.read(bad)
    # the tensor-table entry of "a": name, nd=1, dim 8, type F32, offset
    entry = struct.pack("<Q", 1) + b"a" + struct.pack("<IQI", 1, 8, gguf.T_F32)
    idx = raw.find(entry)
    assert idx > 0
    off_at = idx + len(entry)
    tampered = bytearray(raw)
    tampered[off_at:off_at + 8] = struct.pack("<Q", 4)
    open(bad, "wb").write(bytes(tampered))
    with pytest.raises(gguf.GGUFError, match="not a multiple"):
        gguf.read(bad)
