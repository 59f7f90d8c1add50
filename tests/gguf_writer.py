"""A small GGUF writer for tests (written from the public GGUF v3 layout).

Layout: magic "GGUF", u32 version, u64 tensor count, u64 metadata count;
metadata as (string key, u32 type, value); tensor infos as (string name,
u32 n_dims, u64 dims[n_dims] with dims[0] the contiguous extent, u32 ggml type,
u64 offset relative to the data section); zero padding to the alignment; the
tensor data, each tensor starting on an aligned offset. Strings are a u64
length followed by UTF-8 bytes; arrays are u32 element type, u64 length, elements.
"""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def _value(ty, v) -> bytes:
    if ty == STRING:
        return _str(v)
    if ty == ARRAY:
        ety, items = v
        out = struct.pack("<IQ", ety, len(items))
        for it in items:
            out += _value(ety, it)
        return out
    return struct.pack(_FMT[ty], v)


def gguf_bytes(metadata, tensors, version=3, alignment=None, magic=b"GGUF"):
    """metadata: list of (key, type, value) (arrays: (ARRAY, (elem_type, items)));
    tensors: list of (name, dims (ggml order), ggml_type, raw bytes).
    alignment: written as general.alignment when given (else 32 is used)."""
    align = alignment or 32
    meta = list(metadata)
    if alignment is not None:
        meta.append(("general.alignment", U32, alignment))
    out = bytearray(magic + struct.pack("<IQQ", version, len(tensors), len(meta)))
    for k, ty, v in meta:
        out += _str(k) + struct.pack("<I", ty) + _value(ty, v)
    offsets, off = [], 0
    for _, _, _, raw in tensors:
        offsets.append(off)
        off += (len(raw) + align - 1) // align * align
    for (name, dims, ty, _), o in zip(tensors, offsets):
        out += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", ty, o)
    out += b"\0" * ((-len(out)) % align)
    data_offset = len(out)
    for (_, _, _, raw), o in zip(tensors, offsets):
        assert len(out) == data_offset + o
        out += bytes(raw) + b"\0" * ((-len(raw)) % align)
    return bytes(out), data_offset, offsets


# ggml type ids of the weights the model uses
GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_Q6_K = 0, 1, 8, 12, 14

_NAMES = {10: "attn_norm", 11: "attn_q", 12: "attn_k", 13: "attn_v", 14: "attn_output", 15: "ffn_norm",
          16: "ffn_gate", 17: "ffn_up", 18: "ffn_down"}


def model_gguf(cfg, weights, tie_output=False, f16_norms=False, alignment=None, extra_meta=()):
    """A llama-architecture GGUF of a realm_b200 weights dict
    {(which, layer): (dtype, data)} (dtype ids are ggml's)."""
    H = cfg["hidden"]
    meta = [("general.architecture", STRING, "llama"),
            ("llama.vocab_size", U32, cfg["vocab"]),
            ("llama.embedding_length", U32, H),
            ("llama.block_count", U32, cfg["n_layers"]),
            ("llama.attention.head_count", U32, cfg["n_heads"]),
            ("llama.attention.head_count_kv", U32, cfg["n_kv_heads"]),
            ("llama.feed_forward_length", U32, cfg["ffn"]),
            ("llama.context_length", U32, cfg["max_seq"]),
            ("llama.attention.layer_norm_rms_epsilon", F32, cfg["rms_eps"]),
            ("llama.rope.freq_base", F32, cfg["rope_theta"])] + list(extra_meta)
    tensors = []

    def add(name, dtype, data, rows, cols):
        raw = np.ascontiguousarray(data)
        if dtype == GGML_F32 and f16_norms and rows == 1:
            raw, dtype = np.asarray(raw, np.float32).astype(np.float16), GGML_F16
        dims = [cols] if rows == 1 else [cols, rows]
        tensors.append((name, dims, dtype, raw.view(np.uint8).tobytes()))

    V = cfg["vocab"]
    Q, KV, F = cfg["n_heads"] * cfg["head_dim"], cfg["n_kv_heads"] * cfg["head_dim"], cfg["ffn"]
    shapes = {10: (1, H), 11: (Q, H), 12: (KV, H), 13: (KV, H), 14: (H, Q), 15: (1, H), 16: (F, H), 17: (F, H),
              18: (H, F)}
    add("token_embd.weight", *weights[(0, -1)], V, H)
    add("output_norm.weight", *weights[(1, -1)], 1, H)
    if not tie_output:
        add("output.weight", *weights[(2, -1)], V, H)
    for l in range(cfg["n_layers"]):
        for which, nm in _NAMES.items():
            add(f"blk.{l}.{nm}.weight", *weights[(which, l)], *shapes[which])
    return gguf_bytes(meta, tensors, alignment=alignment)[0]
