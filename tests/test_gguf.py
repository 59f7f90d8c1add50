"""GGUF reader (rb_gguf_*) on CPU: the reference's header test
(crates/realm-core/src/formats/gguf.rs:483-503), round trips of every metadata
type and the tensor dtypes of the decode path, extract_config's keys, fallbacks
and defaults (gguf.rs:214-287), the two size / offset fixes, and corrupt input
(every truncation point and random byte flips fail with an error code)."""
import struct

import numpy as np
import pytest

import gguf_writer as W
import realm_b200 as rb
from realm_b200 import GGUFFile


def test_gguf_magic():
    data = b"GGUF" + struct.pack("<IQQ", 3, 0, 0)
    g = GGUFFile(data=data)
    assert g.version == 3 and g.tensor_count == 0 and g.metadata_kv_count == 0
    assert g.architecture == "unknown" and g.vocab_size is None


def _sample(alignment=None):
    rng = np.random.default_rng(0)
    meta = [
        ("general.architecture", W.STRING, "llama"),
        ("k.u8", W.U8, 250), ("k.i8", W.I8, -7), ("k.u16", W.U16, 65000), ("k.i16", W.I16, -30000),
        ("k.u32", W.U32, 4000000000), ("k.i32", W.I32, -2000000000), ("k.f32", W.F32, 1.5),
        ("k.bool", W.BOOL, 1), ("k.str", W.STRING, "héllo"), ("k.u64", W.U64, 2**63 + 5),
        ("k.i64", W.I64, -(2**62) - 3), ("k.f64", W.F64, 0.1),
        ("k.arr_i32", W.ARRAY, (W.I32, [1, -2, 3])), ("k.arr_f32", W.ARRAY, (W.F32, [0.5, 2.0])),
        ("k.arr_str", W.ARRAY, (W.STRING, ["<s>", "", "▁the"])), ("k.arr_empty", W.ARRAY, (W.U8, [])),
        ("k.arr_bool", W.ARRAY, (W.BOOL, [1, 0, 1])), ("k.empty_str", W.STRING, ""),
    ]
    tensors = [
        ("t.f32", [5, 3], W.GGML_F32, rng.normal(size=15).astype(np.float32).tobytes()),
        ("t.f16", [7], W.GGML_F16, rng.normal(size=7).astype(np.float16).tobytes()),
        ("t.q4k", [512, 2], W.GGML_Q4_K, rng.integers(0, 256, 4 * 144, dtype=np.uint8).tobytes()),
        ("t.q6k", [256, 3], W.GGML_Q6_K, rng.integers(0, 256, 3 * 210, dtype=np.uint8).tobytes()),
        ("t.q80", [64, 5], W.GGML_Q8_0, rng.integers(0, 256, 10 * 34, dtype=np.uint8).tobytes()),
    ]
    data, data_off, offs = W.gguf_bytes(meta, tensors, alignment=alignment)
    return data, data_off, offs, meta, tensors


@pytest.mark.parametrize("alignment", [None, 64, 128])
def test_round_trip_metadata_and_tensors(tmp_path, alignment):
    data, data_off, offs, meta, tensors = _sample(alignment)
    p = tmp_path / "x.gguf"
    p.write_bytes(data)
    for g in (GGUFFile(str(p)), GGUFFile(data=data)):
        assert g.version == 3 and g.data_offset == data_off
        m = g.metadata
        assert m["k.u8"] == 250 and m["k.i8"] == -7 and m["k.u16"] == 65000 and m["k.i16"] == -30000
        assert m["k.u32"] == 4000000000 and m["k.i32"] == -2000000000 and m["k.f32"] == 1.5
        assert m["k.bool"] is True and m["k.str"] == "héllo" and m["k.empty_str"] == ""
        assert m["k.u64"] == 2**63 + 5 and m["k.i64"] == -(2**62) - 3 and m["k.f64"] == 0.1
        assert m["k.arr_i32"].tolist() == [1, -2, 3] and m["k.arr_f32"].tolist() == [0.5, 2.0]
        assert m["k.arr_str"] == ["<s>", "", "▁the"] and m["k.arr_empty"].size == 0
        assert m["k.arr_bool"].tolist() == [True, False, True]
        assert g.architecture == "llama"
        assert [t.name for t in g.tensors] == [t[0] for t in tensors]
        for desc, (name, dims, ty, raw), off in zip(g.tensors, tensors, offs):
            assert desc.dims == tuple(dims) and desc.dtype == ty and desc.offset == off
            assert desc.file_offset == data_off + off and desc.size_bytes == len(raw)
            assert g.tensor_bytes(name).tobytes() == raw
        assert g.tensor("t.q4k").shape == (2, 512)
        with pytest.raises(rb.RealmError) as e:
            g.tensor("nope")
        assert e.value.code == -2 and "Tensor not found: nope" in str(e.value)
        g.close()


def test_size_rules_and_offsets_fix_the_reference():
    """Q8_0 blocks are 34 bytes (tensor.rs:145-150 has 33) and tensor bytes start
    at data section + offset (model_storage.rs:444-464 drops the section offset)."""
    raw = bytes(range(34)) * 4
    data, data_off, offs = W.gguf_bytes([], [("q", [128], W.GGML_Q8_0, raw)])
    g = GGUFFile(data=data)
    t = g.tensors[0]
    assert t.size_bytes == 136 and t.offset == 0 and t.file_offset == data_off > 0
    assert g.tensor_bytes("q").tobytes() == raw


def test_unknown_dtype_parses_with_zero_bytes():
    data, _, _ = W.gguf_bytes([], [("odd", [10], 99, b"\1" * 10)])
    g = GGUFFile(data=data)
    assert g.tensors[0].dtype == 99 and g.tensors[0].size_bytes == 0


@pytest.mark.parametrize("magic,version,msg", [
    (b"GGML", 3, "Invalid GGUF magic: 0x4C4D4747"),
    (b"GGUF", 1, "Unsupported GGUF version: 1"),
    (b"GGUF", 4, "Unsupported GGUF version: 4"),
])
def test_header_errors(magic, version, msg):
    data, _, _ = W.gguf_bytes([], [], version=version, magic=magic)
    with pytest.raises(rb.RealmError) as e:
        GGUFFile(data=data)
    assert e.value.code == -3 and msg in str(e.value)


def test_version_2_is_accepted():
    data, _, _ = W.gguf_bytes([("a", W.U32, 1)], [], version=2)
    assert GGUFFile(data=data).version == 2


def test_value_type_errors():
    bad = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W._str("k") + struct.pack("<I", 13)
    with pytest.raises(rb.RealmError) as e:
        GGUFFile(data=bad)
    assert "Unknown metadata value type: 13" in str(e.value)
    nested = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + W._str("k") + struct.pack("<IIQ", 9, 9, 0)
    with pytest.raises(rb.RealmError) as e:
        GGUFFile(data=nested)
    assert "Unknown typed value: 9" in str(e.value)


def test_tensor_layout_errors():
    data, data_off, _ = W.gguf_bytes([], [("t", [8], W.GGML_F32, b"\0" * 32)])
    with pytest.raises(rb.RealmError) as e:
        GGUFFile(data=data[:-1])                       # tensor runs past the end
    assert e.value.code == -4
    d = bytearray(data)
    info = W._str("t") + struct.pack("<IQIQ", 1, 8, 0, 0)
    i = bytes(d).index(info)
    d[i + len(info) - 8:i + len(info)] = struct.pack("<Q", 4)
    with pytest.raises(rb.RealmError) as e:
        GGUFFile(data=bytes(d))                        # offset not aligned
    assert e.value.code == -3 and "not a multiple" in str(e.value)
    five = b"GGUF" + struct.pack("<IQQ", 3, 1, 0) + W._str("t") + struct.pack("<I", 5)
    with pytest.raises(rb.RealmError) as e:
        GGUFFile(data=five)
    assert "5 dimensions" in str(e.value)
    q4 = W.gguf_bytes([], [("q", [100], W.GGML_Q4_K, b"\0" * 144)])[0]
    with pytest.raises(rb.RealmError) as e:
        GGUFFile(data=q4)                              # 100 is not whole 256-element blocks
    assert e.value.code == -3
    with pytest.raises(rb.RealmError) as e:
        GGUFFile("/nonexistent/x.gguf")
    assert e.value.code == -4


def test_every_truncation_fails_cleanly():
    data, data_off, offs, _, tensors = _sample()
    end = data_off + offs[-1] + len(tensors[-1][3])     # the last tensor byte
    for n in range(end):
        with pytest.raises(rb.RealmError) as e:
            GGUFFile(data=data[:n])
        assert e.value.code in (-3, -4), n
    GGUFFile(data=data[:end]).close()                    # only the final padding missing: fine


def test_invalid_utf8_is_rejected():
    for bad in (b"\xff", b"\xc0\x80", b"\xed\xa0\x80", b"\xe2\x82"):
        d = b"GGUF" + struct.pack("<IQQ", 3, 0, 1) + struct.pack("<Q", len(bad)) + bad + struct.pack("<IB", 0, 1)
        with pytest.raises(rb.RealmError) as e:
            GGUFFile(data=d)
        assert e.value.code == -3 and "Invalid UTF-8" in str(e.value)


def test_random_corruption_never_crashes():
    data, _, _, _, _ = _sample()
    rng = np.random.default_rng(1)
    ok = 0
    for _ in range(400):
        d = bytearray(data)
        for _ in range(int(rng.integers(1, 6))):
            d[int(rng.integers(0, 400))] = int(rng.integers(0, 256))
        try:
            GGUFFile(data=bytes(d)).close()
            ok += 1
        except rb.RealmError as e:
            assert e.code in (-3, -4)
    assert ok < 400


def test_extract_config_keys_fallbacks_and_defaults():
    meta = [("general.architecture", W.STRING, "llama"), ("llama.vocab_size", W.U32, 32000),
            ("llama.embedding_length", W.U32, 4096), ("llama.block_count", W.U32, 32),
            ("llama.attention.head_count", W.U32, 32), ("llama.attention.head_count_kv", W.U32, 8),
            ("llama.feed_forward_length", W.U32, 11008), ("llama.context_length", W.U32, 4096),
            ("llama.attention.layer_norm_rms_epsilon", W.F32, 1e-6), ("llama.rope.freq_base", W.F32, 5e5)]
    c = GGUFFile(data=W.gguf_bytes(meta, [])[0]).model_config()
    assert (c["vocab"], c["hidden"], c["n_layers"], c["n_heads"], c["n_kv_heads"], c["ffn"], c["max_seq"]) == \
        (32000, 4096, 32, 32, 8, 11008, 4096)
    assert c["head_dim"] == 128 and c["rms_eps"] == np.float32(1e-6) and c["layer_eps"] == c["rms_eps"]
    assert c["rope_theta"] == 5e5
    d = GGUFFile(data=W.gguf_bytes([], [])[0]).model_config()   # no keys: the reference's defaults
    assert (d["vocab"], d["hidden"], d["n_layers"], d["n_heads"], d["n_kv_heads"], d["ffn"], d["max_seq"]) == \
        (32000, 2048, 22, 32, 4, 5632, 2048)
    assert d["rms_eps"] == np.float32(1e-5) and d["rope_theta"] == 10000.0 and d["head_dim"] == 64
    alt = [("general.architecture", W.STRING, "qwen"), ("vocab_size", W.I64, 151936),
           ("qwen.hidden_size", W.U16, 1024), ("qwen.num_layers", W.I32, 24), ("rms_norm_eps", W.F64, 1e-6),
           ("qwen.block_count", W.F32, 3.0)]               # float for an integer key: default
    a = GGUFFile(data=W.gguf_bytes(alt, [])[0]).model_config()
    assert a["vocab"] == 151936 and a["hidden"] == 1024 and a["n_layers"] == 22
    assert a["rms_eps"] == np.float32(1e-6)


def test_gguf_null_handles():
    lib = rb.lib()
    assert lib.rb_gguf_version(None) == -20
    assert lib.rb_gguf_tensor_count(None) == -20
    assert lib.rb_model_load_gguf(None, None, None, None) == -20
