"""realm_b200: B200-native decode engine for Realm, host-side Python mirror.

The compute lives in librealm_b200.so (CUDA, sm_100a) behind the C ABI in
include/realm_b200.h. This module binds it with ctypes and mirrors the
reference's (Querent-ai/realm) interfaces for the decode path:

* GpuBackendTrait::fused_dequant_matmul_{q4k,q6k,q80}
  (crates/realm-compute-gpu/src/gpu_backend_trait.rs:17-143)
* the host functions WASM tenants call: candle_matmul(_transposed),
  realm_embed_tokens, realm_forward_layer, realm_compute_logits,
  memory64_load_layer (crates/realm-runtime/src/memory64_host.rs:684-2896)
* KVCache (crates/realm-models/src/kv_cache.rs:7-80) and Model::forward /
  Model::generate (crates/realm-models/src/model.rs:572-847)

There is no CPU fallback: importing fails if the CUDA library is missing, and
every call raises RealmError with the library's status code on failure.
Arrays may be numpy arrays (host) or CUDA torch tensors (device pointers are
passed through without copies).
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "librealm_b200.so")

F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
BLOCK_BYTES = {Q4_K: 144, Q6_K: 210, Q8_0: 34, F32: 4, F16: 2}
BLOCK_ELEMS = {Q4_K: 256, Q6_K: 256, Q8_0: 32, F32: 1, F16: 1}
PTR_HOST, PTR_DEVICE = 0, 1

W_TOKEN_EMBD, W_OUTPUT_NORM, W_OUTPUT = 0, 1, 2
W_ATTN_NORM, W_Q, W_K, W_V, W_O, W_FFN_NORM, W_GATE, W_UP, W_DOWN = range(10, 19)

ERRORS = {
    -1: "feature not available", -2: "not found", -3: "invalid argument / buffer too small",
    -4: "read/write failed", -5: "memory not available", -6: "pointer overflow", -7: "out of bounds",
    -8: "write failed", -20: "bad handle", -21: "KV page pool exhausted", -22: "KV cache overflow",
    -23: "unsupported dtype/shape", -24: "CUDA error", -25: "device wait timed out", -26: "out of device memory",
}

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python realm_b200/build.py` "
                      "(there is no CPU fallback)")

_lib = C.CDLL(LIB_PATH)
_vp, _sz, _u32, _i32, _u64 = C.c_void_p, C.c_size_t, C.c_uint32, C.c_int32, C.c_uint64
_I32P = C.POINTER(C.c_int32)


class _Config(C.Structure):
    _fields_ = [("device", C.c_int32), ("max_rows", C.c_uint32), ("use_pdl", C.c_uint32),
                ("use_graphs", C.c_uint32)]


class _ModelConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim",
                                          "ffn", "vocab", "max_seq")] + [
        ("rms_eps", C.c_float), ("layer_eps", C.c_float), ("rope_theta", C.c_float),
        ("kv_dtype", C.c_int32), ("max_tenants", C.c_uint32), ("kv_pages", C.c_uint32)]


def _sig(name, args, res=C.c_int32):
    f = getattr(_lib, name)
    f.argtypes = args
    f.restype = res
    return f


_sig("rb_ctx_create", [C.POINTER(_Config), C.POINTER(_vp)])
_sig("rb_ctx_destroy", [_vp])
_sig("rb_last_error", [C.c_char_p, _sz])
_sig("rb_sync", [_vp])
_sig("rb_stream", [_vp], _vp)
_sig("rb_num_sms", [_vp])
_sig("rb_kernel_binary_version", [_vp, _I32P])
_sig("rb_test_fail_next_grid_barrier", [_vp, _u32])
_sig("rb_dequantize", [_vp, _i32, _vp, _sz, _vp, _u32])
_sig("rb_quantize", [_vp, _i32, _vp, _sz, _vp, _u32])
_sig("rb_fused_dequant_matmul", [_vp, _i32, _vp, _sz, _vp, _vp, _u32, _u32, _u32, _u32])
_sig("rb_weight_upload", [_vp, _i32, _u32, _u32, _vp, _sz, _u32, _I32P])
_sig("rb_weight_free", [_vp, _i32])
_sig("rb_weight_matmul", [_vp, _i32, _vp, _vp, _u32, _u32])
_sig("rb_weight_export", [_vp, _i32, _vp, _sz, _u32])
_sig("rb_weight_matmul_noalloc", [_vp, _i32, _vp, _vp, _u32, _u32])
_sig("rb_weight_matmul_timing", [_vp, _vp, _u32, _u32, _u32, _u32, C.POINTER(C.c_float)])
_sig("rb_weight_matmul_path", [_vp, _u32])
_sig("rb_candle_matmul", [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32])
_sig("rb_candle_matmul_transposed", [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32])
_sig("rb_kv_pool_create", [_vp, _u32, _u32, _u32, _i32, _u32, _u32, _u32, _I32P])
_sig("rb_kv_pool_destroy", [_vp, _i32])
_sig("rb_kv_pool_shuffle", [_vp, _i32, _u64])
_sig("rb_kv_pool_free_pages", [_vp, _i32])
_sig("rb_kv_create", [_vp, _i32, _u32])
_sig("rb_kv_destroy", [_vp, _i32, _u32])
_sig("rb_kv_clear", [_vp, _i32, _u32])
_sig("rb_kv_len", [_vp, _i32, _u32, _u32])
_sig("rb_kv_append", [_vp, _i32, _u32, _u32, _vp, _vp, _u32, _u32])
_sig("rb_kv_gather", [_vp, _i32, _u32, _u32, _vp, _vp, _u32])
_sig("rb_attention_forward", [_vp, _i32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _u32, C.c_float, _u32])
_sig("rb_model_create", [_vp, C.POINTER(_ModelConfig), _I32P])
_sig("rb_model_destroy", [_vp, _i32])
_sig("rb_model_set_weight", [_vp, _i32, _i32, _i32, _i32, _vp, _sz, _u32])
_sig("rb_model_finalize", [_vp, _i32])
_sig("rb_model_kv_pool", [_vp, _i32])
_sig("rb_tenant_create", [_vp, _i32, _u32])
_sig("rb_tenant_reset", [_vp, _i32, _u32])
_sig("rb_forward", [_vp, _i32, _u32, _vp, _vp, _vp, _vp, _vp, _u32])
_sig("rb_forward_profile", [_vp, _i32, _u32, _vp, _vp, _vp])
_sig("rb_embed_tokens", [_vp, _i32, _vp, _u32, _vp, _u32])
_sig("rb_forward_layer", [_vp, _i32, _u32, _u32, _vp, _u32, _u32, _vp, _u32])
_sig("rb_compute_logits", [_vp, _i32, _vp, _u32, _vp, _u32])
_sig("rb_memory64_load_layer", [_vp, _i32, _u32, _vp, _u32])
_sig("rb_memory64_read", [_vp, _i32, C.c_uint64, _vp, _u32, _u32, _u32, _u32])
_sig("rb_memory64_size", [_vp, _i32, C.POINTER(C.c_uint64)])
_sig("rb_last_forward_ms", [_vp], C.c_float)
_sig("rb_last_forward_launches", [_vp])


class RealmError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}: {ERRORS.get(code, 'error')}] {msg}")
        self.code = code


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    _lib.rb_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def _check(rc: int) -> int:
    if rc < 0:
        raise RealmError(rc, last_error())
    return rc


def lib():
    """The loaded ctypes library (for callers that bind the C ABI directly)."""
    return _lib


# ---- buffer helpers: numpy (host) or torch CUDA tensors (device) ----
def _is_dev(a) -> bool:
    return hasattr(a, "data_ptr") and getattr(a, "is_cuda", False)


def _ptr(a):
    if a is None:
        return None
    if _is_dev(a):
        assert a.is_contiguous()
        return C.c_void_p(a.data_ptr())
    assert isinstance(a, np.ndarray) and a.flags.c_contiguous, "pass contiguous numpy arrays"
    return a.ctypes.data_as(C.c_void_p)


_ORDER_CTX = [None]  # the context whose stream device-tensor calls are ordered on


def _flags(*arrays) -> int:
    devs = [_is_dev(a) for a in arrays if a is not None]
    if any(devs) and not all(devs):
        raise ValueError("mix of host and device buffers in one call")
    if devs and devs[0]:
        # torch produced these tensors on its current stream; make the library's
        # stream wait for that work (stream-ordered, no host synchronisation)
        import torch
        ctx = _ORDER_CTX[0]
        dev = next(a for a in arrays if a is not None).device
        if ctx is not None and ctx._h:
            torch.cuda.ExternalStream(ctx.stream, device=dev).wait_stream(torch.cuda.current_stream(dev))
        return PTR_DEVICE
    return PTR_HOST


def _u8(a):
    return a if _is_dev(a) else np.ascontiguousarray(a).view(np.uint8).ravel()


def _f32(a):
    return a if _is_dev(a) else np.ascontiguousarray(a, dtype=np.float32)


def _u32arr(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.uint32)


class Context:
    """One GPU (rb_ctx). Calls are serialised on the context's stream."""

    def __init__(self, device: int = 0, max_rows: int = 64, pdl: bool = True, graphs: bool = True):
        cfg = _Config(device, max_rows, int(pdl), int(graphs))
        h = _vp()
        _check(_lib.rb_ctx_create(C.byref(cfg), C.byref(h)))
        self._h = h
        self.device = device
        _ORDER_CTX[0] = self

    def close(self):
        if getattr(self, "_h", None) and _lib is not None:
            _lib.rb_ctx_destroy(self._h)
        self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    @property
    def handle(self):
        return self._h

    @property
    def num_sms(self) -> int:
        return _check(_lib.rb_num_sms(self._h))

    @property
    def stream(self) -> int:
        return _lib.rb_stream(self._h)

    def sync(self):
        _check(_lib.rb_sync(self._h))

    def last_forward_ms(self) -> float:
        return float(_lib.rb_last_forward_ms(self._h))

    def last_forward_launches(self) -> int:
        return _check(_lib.rb_last_forward_launches(self._h))

    # ---- quantised blocks ----
    def dequantize(self, dtype: int, blocks, out=None):
        blocks = _u8(blocks)
        nb = (blocks.numel() if _is_dev(blocks) else blocks.nbytes) // BLOCK_BYTES[dtype]
        if out is None:
            out = np.empty(nb * BLOCK_ELEMS[dtype], np.float32)
        _check(_lib.rb_dequantize(self._h, dtype, _ptr(blocks), nb, _ptr(out), _flags(blocks, out)))
        return out

    def quantize(self, dtype: int, x, out=None):
        x = _f32(x)
        n = x.numel() if _is_dev(x) else x.size
        if out is None:
            out = np.empty(n // BLOCK_ELEMS[dtype] * BLOCK_BYTES[dtype], np.uint8)
        _check(_lib.rb_quantize(self._h, dtype, _ptr(x), n, _ptr(out), _flags(x, out)))
        return out

    # ---- GpuBackendTrait::fused_dequant_matmul_* ----
    def fused_dequant_matmul(self, dtype: int, blocks, input, batch_size: int, n: int, k: int, out=None,
                             nblocks: Optional[int] = None):
        blocks = _u8(blocks)
        input = _f32(input)
        if nblocks is None:
            nblocks = (blocks.numel() if _is_dev(blocks) else blocks.nbytes) // BLOCK_BYTES[dtype]
        if out is None:
            out = np.empty((batch_size, n), np.float32)
        _check(_lib.rb_fused_dequant_matmul(self._h, dtype, _ptr(blocks), nblocks, _ptr(input), _ptr(out),
                                            batch_size, n, k, _flags(blocks, input, out)))
        return out

    def fused_dequant_matmul_q4k(self, blocks, input, batch_size, n, k):
        return self.fused_dequant_matmul(Q4_K, blocks, input, batch_size, n, k)

    def fused_dequant_matmul_q6k(self, blocks, input, batch_size, n, k):
        return self.fused_dequant_matmul(Q6_K, blocks, input, batch_size, n, k)

    def fused_dequant_matmul_q80(self, blocks, input, batch_size, n, k):
        return self.fused_dequant_matmul(Q8_0, blocks, input, batch_size, n, k)

    def gemv_timing(self, weights, batch: int, iters: int = 32, reps: int = 5) -> float:
        """Device microseconds per GEMV launch (graph of back-to-back launches)."""
        h = np.array([w.handle for w in weights], np.int32)
        out = C.c_float()
        _check(_lib.rb_weight_matmul_timing(self._h, h.ctypes.data_as(C.c_void_p), len(h), batch, iters, reps,
                                            C.byref(out)))
        return float(out.value)

    def uses_tcgen05(self, batch: int) -> bool:
        """Whether a matmul of `batch` rows runs on the tcgen05 dequant-GEMM."""
        return bool(_lib.rb_weight_matmul_path(self._h, batch))

    def upload_weight(self, dtype: int, n: int, k: int, blocks) -> "Weight":
        return Weight(self, dtype, n, k, blocks)

    # ---- host functions ----
    def candle_matmul(self, a, b, m, k, n, transposed=False, out=None):
        a, b = _f32(a), _f32(b)
        if out is None:
            out = np.empty((m, n), np.float32)
        fn = _lib.rb_candle_matmul_transposed if transposed else _lib.rb_candle_matmul
        _check(fn(self._h, _ptr(a), _ptr(b), _ptr(out), m, k, n, _flags(a, b, out)))
        return out

    def kv_pool(self, n_layers, n_kv_heads, head_dim, kv_dtype=F16, n_pages=1024, max_tenants=64,
                max_seq=8192) -> "KVPool":
        return KVPool(self, n_layers, n_kv_heads, head_dim, kv_dtype, n_pages, max_tenants, max_seq)


class Weight:
    """A [n][k] GGUF weight resident on the device in the tiled GEMV layout."""

    def __init__(self, ctx: Context, dtype: int, n: int, k: int, blocks):
        self.ctx, self.dtype, self.n, self.k = ctx, dtype, n, k
        blocks = _u8(blocks)
        nbytes = blocks.numel() if _is_dev(blocks) else blocks.nbytes
        h = C.c_int32()
        _check(_lib.rb_weight_upload(ctx.handle, dtype, n, k, _ptr(blocks), nbytes, _flags(blocks), C.byref(h)))
        self.handle = h.value

    def matmul(self, x, batch_size: int, out=None):
        x = _f32(x)
        if out is None:
            out = np.empty((batch_size, self.n), np.float32)
        _check(_lib.rb_weight_matmul(self.ctx.handle, self.handle, _ptr(x), _ptr(out), batch_size, _flags(x, out)))
        return out

    def matmul_noalloc(self, x, out, batch_size: int):
        """rb_weight_matmul_noalloc: x [batch][k] and out [batch][n] are CUDA
        tensors owned by the caller; the library allocates nothing for the call
        (batch <= 8, K <= 16384, N <= 131072)."""
        if not (_is_dev(x) and _is_dev(out)):
            raise ValueError("matmul_noalloc takes CUDA tensors only")
        _check(_lib.rb_weight_matmul_noalloc(self.ctx.handle, self.handle, _ptr(x), _ptr(out), batch_size,
                                             _flags(x, out)))
        return out

    def export(self) -> np.ndarray:
        out = np.empty(self.n * (self.k // 256) * 144, np.uint8)
        _check(_lib.rb_weight_export(self.ctx.handle, self.handle, _ptr(out), out.nbytes, PTR_HOST))
        return out

    def free(self):
        if self.handle >= 0:
            _check(_lib.rb_weight_free(self.ctx.handle, self.handle))
            self.handle = -1


class KVPool:
    """Paged KV pool (16-token pages for all layers of one geometry)."""

    def __init__(self, ctx, n_layers, n_kv_heads, head_dim, kv_dtype, n_pages, max_tenants, max_seq,
                 handle: Optional[int] = None):
        self.ctx = ctx
        self.n_layers, self.n_kv, self.hd, self.kv_dtype = n_layers, n_kv_heads, head_dim, kv_dtype
        self.max_seq = max_seq
        if handle is None:
            h = C.c_int32()
            _check(_lib.rb_kv_pool_create(ctx.handle, n_layers, n_kv_heads, head_dim, kv_dtype, n_pages,
                                          max_tenants, max_seq, C.byref(h)))
            handle = h.value
        self.handle = handle

    def shuffle(self, seed: int):
        _check(_lib.rb_kv_pool_shuffle(self.ctx.handle, self.handle, seed))

    def free_pages(self) -> int:
        return _check(_lib.rb_kv_pool_free_pages(self.ctx.handle, self.handle))

    def create(self, tenant: int):
        _check(_lib.rb_kv_create(self.ctx.handle, self.handle, tenant))

    def destroy(self, tenant: int):
        _check(_lib.rb_kv_destroy(self.ctx.handle, self.handle, tenant))

    def clear(self, tenant: int):
        _check(_lib.rb_kv_clear(self.ctx.handle, self.handle, tenant))

    def len(self, tenant: int, layer: int = 0) -> int:
        return _check(_lib.rb_kv_len(self.ctx.handle, self.handle, tenant, layer))

    def append(self, tenant: int, layer: int, k, v) -> int:
        k, v = _f32(k), _f32(v)
        n = k.numel() if _is_dev(k) else k.size
        seq = n // (self.n_kv * self.hd)
        return _check(_lib.rb_kv_append(self.ctx.handle, self.handle, tenant, layer, _ptr(k), _ptr(v), seq,
                                         _flags(k, v)))

    def gather(self, tenant: int, layer: int):
        n = self.len(tenant, layer) * self.n_kv * self.hd
        k = np.empty(n, np.float32)
        v = np.empty(n, np.float32)
        if n:
            _check(_lib.rb_kv_gather(self.ctx.handle, self.handle, tenant, layer, _ptr(k), _ptr(v), PTR_HOST))
        return k, v

    def attention_forward(self, layer: int, tenants: Sequence[int], q, n_heads: int, scale: float,
                          positions=None, k_new=None, v_new=None, out=None):
        """Paged decode attention (the north star's attention_forward)."""
        t = _u32arr(tenants)
        p = _u32arr(positions)
        q = _f32(q)
        k_new = None if k_new is None else _f32(k_new)
        v_new = None if v_new is None else _f32(v_new)
        if out is None:
            out = np.empty((len(t), n_heads * self.hd), np.float32)
        _check(_lib.rb_attention_forward(self.ctx.handle, self.handle, layer, len(t), _ptr(t), _ptr(p), _ptr(q),
                                         _ptr(k_new), _ptr(v_new), _ptr(out), n_heads, scale,
                                         _flags(q, k_new, v_new, out)))
        return out


class KVCache:
    """Mirror of realm_models::KVCache for one tenant and one layer
    (crates/realm-models/src/kv_cache.rs:7-80) on a private paged pool."""

    def __init__(self, ctx: Context, max_seq_len: int, num_kv_heads: int, head_dim: int, kv_dtype: int = F32):
        pages = (max_seq_len + 15) // 16
        self.pool = KVPool(ctx, 1, num_kv_heads, head_dim, kv_dtype, pages, 1, max_seq_len)
        self.pool.create(0)
        self.max_seq_len, self.num_kv_heads, self.head_dim = max_seq_len, num_kv_heads, head_dim

    @property
    def current_seq_len(self) -> int:
        return self.pool.len(0, 0)

    def append(self, keys, values):
        """Appends and, like the reference, returns copies of the whole cached prefix."""
        self.pool.append(0, 0, keys, values)
        return self.current_data()

    def current_data(self):
        return self.pool.gather(0, 0)

    def clear(self):
        self.pool.clear(0)


class Model:
    """Device-resident transformer (Llama family) with per-tenant paged KV.

    cfg keys: n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab,
    max_seq, rms_eps, layer_eps, rope_theta, kv_dtype (F16/F32), max_tenants,
    kv_pages (optional).
    """

    def __init__(self, ctx: Context, cfg: dict):
        self.ctx, self.cfg = ctx, dict(cfg)
        c = _ModelConfig(cfg["n_layers"], cfg["hidden"], cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"],
                         cfg["ffn"], cfg["vocab"], cfg["max_seq"], cfg["rms_eps"], cfg["layer_eps"],
                         cfg["rope_theta"], cfg.get("kv_dtype", F16), cfg.get("max_tenants", 64),
                         cfg.get("kv_pages", 0))
        h = C.c_int32()
        _check(_lib.rb_model_create(ctx.handle, C.byref(c), C.byref(h)))
        self.handle = h.value
        pool = _check(_lib.rb_model_kv_pool(ctx.handle, self.handle))
        self.kv = KVPool(ctx, cfg["n_layers"], cfg["n_kv_heads"], cfg["head_dim"], cfg.get("kv_dtype", F16), 0, 0,
                         cfg["max_seq"], handle=pool)

    @classmethod
    def attach(cls, ctx: Context, cfg: dict, handle: int) -> "Model":
        """Wraps a model the library created (e.g. rb_model_load_gguf)."""
        m = cls.__new__(cls)
        m.ctx, m.cfg, m.handle = ctx, dict(cfg), handle
        pool = _check(_lib.rb_model_kv_pool(ctx.handle, handle))
        m.kv = KVPool(ctx, cfg["n_layers"], cfg["n_kv_heads"], cfg["head_dim"], cfg.get("kv_dtype", F16), 0, 0,
                      cfg["max_seq"], handle=pool)
        return m

    def set_weight(self, which: int, layer: int, dtype: int, data):
        if not _is_dev(data):
            if dtype == F32:
                data = np.ascontiguousarray(data, np.float32)
            data = np.ascontiguousarray(data).view(np.uint8).ravel()
        nbytes = (data.numel() * data.element_size()) if _is_dev(data) else data.nbytes
        _check(_lib.rb_model_set_weight(self.ctx.handle, self.handle, which, layer, dtype, _ptr(data), nbytes,
                                        _flags(data)))

    def set_weights(self, weights: dict):
        for (which, layer), (dtype, data) in weights.items():
            self.set_weight(which, layer, dtype, data)
        self.finalize()

    def finalize(self):
        _check(_lib.rb_model_finalize(self.ctx.handle, self.handle))

    def tenant_create(self, tenant: int):
        _check(_lib.rb_tenant_create(self.ctx.handle, self.handle, tenant))

    def tenant_reset(self, tenant: int):
        _check(_lib.rb_tenant_reset(self.ctx.handle, self.handle, tenant))

    def forward_rows(self, tenants, tokens, positions=None, want_logits=True):
        """Batched forward; returns (logits [n][vocab] or None, argmax [n])."""
        t = _u32arr(tenants)
        tok = _u32arr(tokens)
        p = _u32arr(positions)
        n = len(t)
        logits = np.empty((n, self.cfg["vocab"]), np.float32) if want_logits else None
        am = np.empty(n, np.uint32)
        _check(_lib.rb_forward(self.ctx.handle, self.handle, n, _ptr(t), _ptr(tok), _ptr(p), _ptr(logits), _ptr(am),
                               PTR_HOST))
        return logits, am

    def forward_profile(self, tenants, tokens):
        """One decode step run kernel by kernel (no graph, no overlap): summed
        device ms of the embedding, GEMV chain, attention and tcgen05 GEMM
        launches, and the launch count."""
        t = _u32arr(tenants)
        tok = _u32arr(tokens)
        ms = np.zeros(4, np.float32)
        n = _check(_lib.rb_forward_profile(self.ctx.handle, self.handle, len(t), _ptr(t), _ptr(tok), _ptr(ms)))
        return dict(zip(("embed", "gemv", "attention", "qgemm"), ms.tolist())), n

    def forward(self, token_ids, position: int, tenant: int = 0):
        """Model::forward (model.rs:572-625): logits of the last token."""
        ids = list(token_ids)
        logits, _ = self.forward_rows([tenant] * len(ids), ids, [position + i for i in range(len(ids))])
        return logits[-1]

    def generate(self, prompt, max_tokens: int, tenant: int = 0, chunk: int = 8, want_logits=False):
        """Model::generate greedy path (model.rs:749-847): prefill in 8-token chunks, then decode."""
        self.tenant_create(tenant)
        prompt = list(prompt)
        out, step_logits = [], []
        for cs in range(0, len(prompt), chunk):
            ids = prompt[cs:cs + chunk]
            lg, am = self.forward_rows([tenant] * len(ids), ids, want_logits=want_logits)
        for g in range(max_tokens):
            if g > 0:
                lg, am = self.forward_rows([tenant], [out[-1]], want_logits=want_logits)
            out.append(int(am[-1]))
            if want_logits:
                step_logits.append(lg[-1].copy())
        return np.array(out, np.uint32), (np.stack(step_logits) if want_logits else None)

    # ---- host-function mirrors ----
    def realm_embed_tokens(self, token_ids):
        ids = _u32arr(token_ids)
        out = np.empty((len(ids), self.cfg["hidden"]), np.float32)
        _check(_lib.rb_embed_tokens(self.ctx.handle, self.handle, _ptr(ids), len(ids), _ptr(out), PTR_HOST))
        return out

    def realm_forward_layer(self, tenant: int, layer: int, hidden, position: int):
        hidden = np.ascontiguousarray(hidden, np.float32)
        out = np.empty_like(hidden)
        _check(_lib.rb_forward_layer(self.ctx.handle, self.handle, tenant, layer, _ptr(hidden), hidden.size,
                                     position, _ptr(out), PTR_HOST))
        return out

    def realm_compute_logits(self, hidden):
        hidden = np.ascontiguousarray(hidden, np.float32).ravel()
        out = np.empty(self.cfg["vocab"], np.float32)
        _check(_lib.rb_compute_logits(self.ctx.handle, self.handle, _ptr(hidden), hidden.size, _ptr(out), PTR_HOST))
        return out

    def memory64_load_layer(self, layer_id: int, max_size: int) -> np.ndarray:
        buf = np.empty(max_size, np.uint8)
        n = _check(_lib.rb_memory64_load_layer(self.ctx.handle, self.handle, layer_id, _ptr(buf), max_size))
        return buf[:n]

    def memory64_size(self) -> int:
        n = C.c_uint64()
        _check(_lib.rb_memory64_size(self.ctx.handle, self.handle, C.byref(n)))
        return n.value

    def memory64_read(self, offset: int, mem, mem_offset: int, size: int) -> int:
        """memory64_read: `size` bytes at `offset` of the Memory64 image into the
        caller's linear memory `mem` (a uint8 array or CUDA tensor) at mem_offset."""
        nbytes = (mem.numel() * mem.element_size()) if _is_dev(mem) else mem.nbytes
        return _check(_lib.rb_memory64_read(self.ctx.handle, self.handle, offset, _ptr(mem), nbytes, mem_offset,
                                            size, _flags(mem)))

    def close(self):
        if self.handle >= 0:
            _lib.rb_model_destroy(self.ctx.handle, self.handle)
            self.handle = -1


from .batching import (BatchedRequest, BatchStats, ContinuousBatcher, Scheduler,  # noqa: E402
                       prepare_batch)
from .gguf import GGUFFile, TensorDesc  # noqa: E402
from .sampling import LogitsProcessor, SamplingParams, sample_logits, sampling_uniform  # noqa: E402
