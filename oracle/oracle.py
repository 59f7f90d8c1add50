"""ctypes wrapper over the C++ CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker and the timed CPU baseline. The
product package (realm_b200) never imports this module; only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline legs do.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

F32, F16, Q80, Q4K, Q6K = 0, 1, 8, 12, 14
BLOCK_BYTES = {Q4K: 144, Q6K: 210, Q80: 34, F32: 4, F16: 2}
BLOCK_ELEMS = {Q4K: 256, Q6K: 256, Q80: 32, F32: 1, F16: 1}

W_TOKEN_EMBD, W_OUTPUT_NORM, W_OUTPUT = 0, 1, 2
W_ATTN_NORM, W_Q, W_K, W_V, W_O, W_FFN_NORM, W_GATE, W_UP, W_DOWN = range(10, 19)


def build() -> str:
    """Compile liboracle.so with the committed Makefile (no-op when up to date)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        vp, sz, fp, i32 = C.c_void_p, C.c_size_t, C.POINTER(C.c_float), C.c_int
        L.or_dequant.argtypes = [i32, vp, sz, vp]
        L.or_quantize.argtypes = [i32, vp, sz, vp]
        L.or_fused_matmul.argtypes = [i32, vp, sz, vp, vp, sz, sz, sz, i32]
        L.or_dequant_matmul.argtypes = [i32, vp, sz, vp, vp, sz, sz, sz, i32]
        L.or_dequant_matmul_scalar.argtypes = [i32, vp, sz, vp, vp, sz, sz, sz, i32]
        L.or_dequant_matmul_f64.argtypes = [i32, vp, sz, vp, vp, sz, sz, sz, i32]
        L.or_rms_norm.argtypes = [vp, vp, C.c_float, sz, sz, vp]
        L.or_rope.argtypes = [vp, sz, sz, sz, sz, C.c_float]
        L.or_attention.argtypes = [vp, vp, vp, sz, sz, sz, sz, sz, sz, vp]
        L.or_sample.argtypes = [vp, sz, C.c_double, C.c_double, sz, C.c_float, vp, sz, C.c_float, vp]
        L.or_kv_new.argtypes = [sz, sz, sz, i32]
        L.or_kv_new.restype = vp
        L.or_kv_free.argtypes = [vp]
        L.or_kv_append.argtypes = [vp, vp, vp, sz]
        L.or_kv_len.argtypes = [vp]
        L.or_kv_len.restype = sz
        L.or_kv_data.argtypes = [vp, vp, vp]
        L.or_kv_clear.argtypes = [vp]
        L.or_model_new.argtypes = [vp]
        L.or_model_new.restype = vp
        L.or_model_free.argtypes = [vp]
        L.or_model_set_weight.argtypes = [vp, i32, i32, i32, vp, sz]
        L.or_model_forward.argtypes = [vp, vp, sz, sz, vp]
        L.or_model_last_hidden.argtypes = [vp, vp]
        L.or_model_clear_kv.argtypes = [vp]
        L.or_model_kv_fill.argtypes = [vp, sz, C.c_uint64]
        L.or_model_kv_len.argtypes = [vp, i32]
        L.or_model_kv_len.restype = sz
        L.or_model_kv_data.argtypes = [vp, i32, vp, vp]
        L.or_model_generate.argtypes = [vp, vp, sz, sz, vp, vp]
        L.or_argmax.argtypes = [vp, sz]
        L.or_argmax.restype = C.c_uint32
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_f16_to_f32.restype = C.c_float
        L.or_f32_to_f16.argtypes = [C.c_float]
        L.or_f32_to_f16.restype = C.c_uint16
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags.c_contiguous
    return a.ctypes.data_as(C.c_void_p)


def nblocks(dtype: int, nbytes: int) -> int:
    return nbytes // BLOCK_BYTES[dtype]


def dequant(dtype: int, blocks: np.ndarray) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    nb = nblocks(dtype, blocks.nbytes)
    out = np.empty(nb * BLOCK_ELEMS[dtype], np.float32)
    rc = lib().or_dequant(dtype, _p(blocks), nb, _p(out))
    assert rc == 0, rc
    return out


def quantize(dtype: int, x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32).ravel()
    be = BLOCK_ELEMS[dtype]
    assert x.size % be == 0
    out = np.empty(x.size // be * BLOCK_BYTES[dtype], np.uint8)
    rc = lib().or_quantize(dtype, _p(x), x.size, _p(out))
    assert rc == 0, rc
    return out


def fused_matmul(dtype, blocks, x, m, n, k, threads=1, nblocks_override=None):
    """Reference fused_dequant_matmul_* (fused.rs) -> (rc, y[m, n])."""
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros((m, n), np.float32)
    nb = nblocks(dtype, blocks.nbytes) if nblocks_override is None else nblocks_override
    rc = lib().or_fused_matmul(dtype, _p(blocks), nb, _p(x), _p(y), m, n, k, threads)
    return rc, y


def dequant_matmul(dtype, blocks, x, m, n, k, threads=0, f64=False, scalar=False):
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros((m, n), np.float64 if f64 else np.float32)
    fn = (lib().or_dequant_matmul_f64 if f64 else
          lib().or_dequant_matmul_scalar if scalar else lib().or_dequant_matmul)
    rc = fn(dtype, _p(blocks), nblocks(dtype, blocks.nbytes), _p(x), _p(y), m, n, k, threads)
    assert rc >= 0, rc
    return y


def rms_norm(x, w, eps):
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    y = np.empty_like(x)
    lib().or_rms_norm(_p(x), _p(w), eps, x.shape[0], x.shape[1], _p(y))
    return y


def rope(t, start_pos, seq_len, n_heads, hd, theta):
    t = np.array(t, np.float32, copy=True)
    lib().or_rope(_p(t), start_pos, seq_len, n_heads, hd, theta)
    return t


def attention(q, k, v, seq_len, kv_len, position, n_heads, n_kv, hd):
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.zeros(seq_len * n_heads * hd, np.float32)
    lib().or_attention(_p(q), _p(k), _p(v), seq_len, kv_len, position, n_heads, n_kv, hd, _p(out))
    return out


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().or_argmax(_p(x), x.size))


def sample(logits, temperature, top_p, top_k, penalty, prev, u):
    """LogitsProcessor::with_params(..).sample (sampling.rs:63-300) with the uniform
    draw u supplied; returns (token or None on the reference's Err, penalised logits)."""
    x = np.array(logits, np.float32)
    pv = np.ascontiguousarray(np.asarray(prev, np.int64).astype(np.uint32))
    out = np.zeros(1, np.uint32)
    rc = lib().or_sample(_p(x), x.size, float(temperature), float(top_p), int(top_k), float(penalty),
                         _p(pv) if pv.size else None, pv.size, float(u), _p(out))
    return (None if rc < 0 else int(out[0])), x


def f32_to_f16_bits(v: float) -> int:
    return int(lib().or_f32_to_f16(v))


class KVCache:
    """crates/realm-models/src/kv_cache.rs:7-80 (kv_fp16 rounds K/V to fp16 on append)."""

    def __init__(self, max_seq, n_kv, hd, kv_fp16=False):
        self.n_kv, self.hd = n_kv, hd
        self._h = lib().or_kv_new(max_seq, n_kv, hd, int(kv_fp16))

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_kv_free(self._h)
            self._h = None

    def append(self, k, v) -> int:
        k = np.ascontiguousarray(k, np.float32)
        v = np.ascontiguousarray(v, np.float32)
        return lib().or_kv_append(self._h, _p(k), _p(v), k.size)

    @property
    def current_seq_len(self):
        return int(lib().or_kv_len(self._h))

    def current_data(self):
        n = self.current_seq_len * self.n_kv * self.hd
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        lib().or_kv_data(self._h, _p(k), _p(v))
        return k, v

    def clear(self):
        lib().or_kv_clear(self._h)


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim",
                                         "ffn", "vocab", "max_seq")] + [
        ("rms_eps", C.c_float), ("layer_eps", C.c_float), ("rope_theta", C.c_float),
        ("kv_fp16", C.c_int32), ("threads", C.c_int32)]


class Model:
    """realm_models::Model restated (model.rs:572-847) over quantised weights."""

    def __init__(self, cfg: dict, weights: dict, threads: int = 0):
        self.cfg = cfg
        c = _Cfg(cfg["n_layers"], cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                 cfg["ffn"], cfg["vocab"], cfg["max_seq"], cfg["rms_eps"], cfg["layer_eps"],
                 cfg["rope_theta"], int(cfg.get("kv_fp16", 0)), threads)
        self._h = lib().or_model_new(C.byref(c))
        for (which, layer), (dtype, data) in weights.items():
            data = np.ascontiguousarray(data).view(np.uint8)
            rc = lib().or_model_set_weight(self._h, which, layer, dtype, _p(data), data.nbytes)
            assert rc >= 0, (which, layer, rc)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().or_model_free(self._h)
            self._h = None

    def forward(self, tokens, position):
        t = np.ascontiguousarray(tokens, np.uint32)
        logits = np.empty(self.cfg["vocab"], np.float32)
        rc = lib().or_model_forward(self._h, _p(t), t.size, position, _p(logits))
        assert rc >= 0, rc
        return logits

    def last_hidden(self):
        h = np.empty(self.cfg["hidden"], np.float32)
        lib().or_model_last_hidden(self._h, _p(h))
        return h

    def clear_kv(self):
        lib().or_model_clear_kv(self._h)

    def kv_fill(self, n, seed=0):
        rc = lib().or_model_kv_fill(self._h, n, seed)
        assert rc >= 0, rc

    def kv_len(self, layer=0):
        return int(lib().or_model_kv_len(self._h, layer))

    def kv_data(self, layer):
        n = self.kv_len(layer) * self.cfg["n_kv_heads"] * self.cfg["head_dim"]
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        lib().or_model_kv_data(self._h, layer, _p(k), _p(v))
        return k, v

    def generate(self, prompt, n_gen, want_logits=True):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.empty(n_gen, np.uint32)
        logits = np.empty((n_gen, self.cfg["vocab"]), np.float32) if want_logits else None
        rc = lib().or_model_generate(self._h, _p(p), p.size, n_gen, _p(out),
                                     _p(logits) if want_logits else None)
        assert rc >= 0, rc
        return out, logits
