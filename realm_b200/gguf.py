"""GGUF files: GGUFParser (crates/realm-core/src/formats/gguf.rs:100-479) over the
native reader (rb_gguf_*), and Model::load_from_gguf
(crates/realm-models/src/model.rs:291-540) onto the device (rb_model_load_gguf).

The file is memory-mapped by the library; tensor bytes are uploaded from the
mapping without a host copy. ``metadata`` decodes every key/value into Python
values (numeric arrays as numpy arrays, string arrays as lists of str).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import F16, _check, _lib, _ModelConfig, _sig, Model

_vp, _u32, _i32, _u64, _i64 = C.c_void_p, C.c_uint32, C.c_int32, C.c_uint64, C.c_int64

U8, I8, U16, I16, U32, I32, F32_, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_NP = {U8: np.uint8, I8: np.int8, U16: np.uint16, I16: np.int16, U32: np.uint32, I32: np.int32, F32_: np.float32,
       BOOL: np.uint8, U64: np.uint64, I64: np.int64, F64: np.float64}


class _Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int32), ("n_dims", C.c_uint32), ("dims", C.c_uint64 * 4),
                ("offset", C.c_uint64), ("file_offset", C.c_uint64), ("nbytes", C.c_uint64), ("data", C.c_void_p)]


_sig("rb_gguf_open", [C.c_char_p, C.POINTER(_vp)])
_sig("rb_gguf_open_memory", [_vp, C.c_size_t, C.POINTER(_vp)])
_sig("rb_gguf_close", [_vp])
_sig("rb_gguf_version", [_vp])
_sig("rb_gguf_data_offset", [_vp, C.POINTER(_u64)])
_sig("rb_gguf_tensor_count", [_vp])
_sig("rb_gguf_tensor_info", [_vp, _u32, C.POINTER(_Tensor)])
_sig("rb_gguf_find_tensor", [_vp, C.c_char_p])
_sig("rb_gguf_meta_count", [_vp])
_sig("rb_gguf_meta_entry", [_vp, _u32, C.POINTER(C.c_char_p), C.POINTER(_i32), C.POINTER(_i32), C.POINTER(_u64)])
_sig("rb_gguf_meta_find", [_vp, C.c_char_p])
_sig("rb_gguf_meta_u32", [_vp, _u32, C.POINTER(_u32)])
_sig("rb_gguf_meta_f32", [_vp, _u32, C.POINTER(C.c_float)])
_sig("rb_gguf_meta_scalar", [_vp, _u32, _vp, C.c_size_t])
_sig("rb_gguf_meta_string", [_vp, _u32, _i64, C.POINTER(_vp), C.POINTER(_u64)])
_sig("rb_gguf_meta_array_data", [_vp, _u32, C.POINTER(_vp)])
_sig("rb_gguf_model_config", [_vp, C.POINTER(_ModelConfig)])
_sig("rb_model_load_gguf", [_vp, _vp, C.POINTER(_ModelConfig), C.POINTER(_i32)])


@dataclass
class TensorDesc:
    """TensorDesc (crates/realm-core/src/tensor.rs:116-193) plus where its bytes are."""
    name: str
    dtype: int
    dims: Tuple[int, ...]        # ggml order: dims[0] is the contiguous extent
    offset: int                  # relative to the data section, as stored
    file_offset: int
    size_bytes: int

    @property
    def shape(self) -> Tuple[int, ...]:
        """Row-major shape (outermost first): [vocab, hidden] for token_embd."""
        return tuple(reversed(self.dims))


class GGUFFile:
    """A parsed GGUF file (GGUFParser::parse_header's ModelMeta, gguf.rs:87-97)."""

    def __init__(self, path: Optional[str] = None, data: Optional[bytes] = None):
        h = _vp()
        if path is not None:
            _check(_lib.rb_gguf_open(str(path).encode(), C.byref(h)))
            self._buf = None
        else:
            self._buf = np.frombuffer(bytes(data), np.uint8)  # kept alive: the handle points into it
            _check(_lib.rb_gguf_open_memory(self._buf.ctypes.data if self._buf.size else None, self._buf.size,
                                            C.byref(h)))
        self._h = h
        self.version = _check(_lib.rb_gguf_version(h))
        off = _u64()
        _check(_lib.rb_gguf_data_offset(h, C.byref(off)))
        self.data_offset = int(off.value)
        self.tensors: List[TensorDesc] = []
        t = _Tensor()
        for i in range(_check(_lib.rb_gguf_tensor_count(h))):
            _check(_lib.rb_gguf_tensor_info(h, i, C.byref(t)))
            self.tensors.append(TensorDesc(t.name.decode(), int(t.dtype), tuple(int(d) for d in t.dims[:t.n_dims]),
                                           int(t.offset), int(t.file_offset), int(t.nbytes)))
        self.metadata: Dict[str, object] = {}
        self.metadata_types: Dict[str, int] = {}
        for i in range(_check(_lib.rb_gguf_meta_count(h))):
            key, ty, ety, n = C.c_char_p(), _i32(), _i32(), _u64()
            _check(_lib.rb_gguf_meta_entry(h, i, C.byref(key), C.byref(ty), C.byref(ety), C.byref(n)))
            k = key.value.decode()
            self.metadata[k] = self._value(i, ty.value, ety.value, n.value)
            self.metadata_types[k] = ty.value

    def _string(self, i, elem=-1) -> str:
        p, n = _vp(), _u64()
        _check(_lib.rb_gguf_meta_string(self._h, i, elem, C.byref(p), C.byref(n)))
        return C.string_at(p.value, n.value).decode("utf-8") if n.value else ""

    def _value(self, i, ty, ety, n):
        if ty == STRING:
            return self._string(i)
        if ty == ARRAY:
            if ety == STRING:
                return [self._string(i, j) for j in range(n)]
            p = _vp()
            _check(_lib.rb_gguf_meta_array_data(self._h, i, C.byref(p)))
            dt = _NP[ety]
            a = np.frombuffer(C.string_at(p.value, n * np.dtype(dt).itemsize), dt).copy() if n else np.zeros(0, dt)
            return a.astype(bool) if ety == BOOL else a
        raw = C.create_string_buffer(8)
        nb = _check(_lib.rb_gguf_meta_scalar(self._h, i, raw, 8))
        v = np.frombuffer(raw.raw[:nb], _NP[ty])[0]
        if ty == BOOL:
            return bool(v)
        return float(v) if ty in (F32_, F64) else int(v)

    def close(self):
        if getattr(self, "_h", None):
            _lib.rb_gguf_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    # ---- ModelMeta fields ----
    @property
    def tensor_count(self) -> int:
        return len(self.tensors)

    @property
    def metadata_kv_count(self) -> int:
        return len(self.metadata)

    @property
    def architecture(self) -> str:
        a = self.metadata.get("general.architecture")
        return a if isinstance(a, str) else "unknown"

    @property
    def vocab_size(self) -> Optional[int]:
        i = self._find_meta(f"{self.architecture}.vocab_size")
        if i is None:
            i = self._find_meta("vocab_size")
        if i is None:
            return None
        v = _u32()
        return int(v.value) if _lib.rb_gguf_meta_u32(self._h, i, C.byref(v)) == 0 else None

    def _find_meta(self, key):
        i = _lib.rb_gguf_meta_find(self._h, key.encode())
        return None if i < 0 else i

    def tensor(self, name: str) -> TensorDesc:
        return self.tensors[_check(_lib.rb_gguf_find_tensor(self._h, name.encode()))]

    def tensor_bytes(self, name: str) -> np.ndarray:
        """A host copy of a tensor's bytes (read through the mapping)."""
        t = _Tensor()
        _check(_lib.rb_gguf_tensor_info(self._h, _check(_lib.rb_gguf_find_tensor(self._h, name.encode())),
                                        C.byref(t)))
        return np.frombuffer(C.string_at(t.data, t.nbytes), np.uint8).copy()

    def model_config(self) -> dict:
        """extract_config (gguf.rs:214-287) as the dict realm_b200.Model takes."""
        c = _ModelConfig()
        _check(_lib.rb_gguf_model_config(self._h, C.byref(c)))
        return {n: getattr(c, n) for n, _ in _ModelConfig._fields_}

    def load_model(self, ctx, kv_dtype: int = F16, max_tenants: int = 64, kv_pages: int = 0,
                   max_seq: Optional[int] = None, **overrides) -> Model:
        """Model::load_from_gguf onto the device. The geometry comes from
        model_config(); vocab follows token_embd.weight when the file has no
        vocab_size key (the reference would assume 32000)."""
        cfg = self.model_config()
        if self.vocab_size is None:
            try:
                cfg["vocab"] = self.tensor("token_embd.weight").dims[1]
            except Exception:
                pass
        cfg.update(kv_dtype=kv_dtype, max_tenants=max_tenants, kv_pages=kv_pages)
        if max_seq is not None:
            cfg["max_seq"] = max_seq
        cfg.update(overrides)
        c = _ModelConfig(*[cfg[n] for n, _ in _ModelConfig._fields_])
        h = _i32()
        _check(_lib.rb_model_load_gguf(ctx.handle, self._h, C.byref(c), C.byref(h)))
        return Model.attach(ctx, cfg, h.value)
