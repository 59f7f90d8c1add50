"""Sampling: LogitsProcessor (crates/realm-models/src/sampling.rs) on the device.

``LogitsProcessor.with_params / new / from_sampling`` pick the strategy as the
reference does (sampling.rs:37-100); ``sample(logits)`` runs the fused kernel
(rb_sample_logits): repetition penalty over the processor's own previous
tokens, temperature, softmax, top-k, top-p and a WeightedIndex draw. The
uniform draws come from ``sampling_uniform(seed, i)`` for the processor's i-th
sample (a counter-based stream on the same 2^-23 grid as rand 0.8.5's f32
sampler; the reference's StdRng stream itself is not reproduced).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

from . import _check, _lib, _sig

_vp, _u32, _u64 = C.c_void_p, C.c_uint32, C.c_uint64


class _Sampling(C.Structure):
    _fields_ = [("temperature", C.c_double), ("top_p", C.c_double), ("top_k", C.c_uint32),
                ("repetition_penalty", C.c_float)]


_sig("rb_sample_logits", [_vp, _vp, _u32, _u32, _u32, _vp, _vp, _vp, _vp, _vp, _u32])
_sig("rb_sampling_uniform", [_u64, _u64], C.c_float)
_sig("rb_forward_sample", [_vp, C.c_int32, _u32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp])


@dataclass
class SamplingParams:
    """The with_params arguments (sampling.rs:63-100)."""
    temperature: float = 0.0
    top_p: float = 1.0
    top_k: int = 0
    repetition_penalty: float = 1.0

    def c(self) -> _Sampling:
        return _Sampling(float(self.temperature), float(self.top_p), int(self.top_k), float(self.repetition_penalty))


def sampling_uniform(seed: int, counter: int) -> float:
    return float(_lib.rb_sampling_uniform(seed & (2**64 - 1), counter & (2**64 - 1)))


def _params_array(params: Sequence[SamplingParams]):
    arr = (_Sampling * len(params))()
    for i, p in enumerate(params):
        arr[i] = p.c()
    return arr


def _prev_arrays(prev: Optional[Sequence[Sequence[int]]], n: int):
    if prev is None:
        return None, None
    off = np.zeros(n + 1, np.uint32)
    flat: List[int] = []
    for r in range(n):
        off[r] = len(flat)
        flat.extend(int(t) for t in prev[r])
    off[n] = len(flat)
    return np.array(flat or [0], np.uint32), off


def sample_logits(ctx, logits, params: Sequence[SamplingParams], uniforms, prev=None) -> np.ndarray:
    """One token per row of host logits [n][vocab] (numpy); prev: per-row previous tokens."""
    x = np.ascontiguousarray(logits, np.float32)
    if x.ndim == 1:
        x = x[None]
    n, v = x.shape
    u = np.ascontiguousarray(uniforms, np.float32).reshape(n)
    pflat, poff = _prev_arrays(prev, n)
    out = np.empty(n, np.uint32)
    _check(_lib.rb_sample_logits(ctx.handle, x.ctypes.data, v, n, v, _params_array(params),
                                 pflat.ctypes.data if pflat is not None else None,
                                 poff.ctypes.data if poff is not None else None, u.ctypes.data, out.ctypes.data, 0))
    return out


class LogitsProcessor:
    """LogitsProcessor (sampling.rs:28-300) over the device kernel."""

    def __init__(self, ctx, seed: int, params: SamplingParams):
        self.ctx, self.seed, self.params = ctx, seed, params
        self.previous_tokens: List[int] = []

    @classmethod
    def with_params(cls, ctx, seed: int, temperature: float, top_p: float, top_k: int,
                    repetition_penalty: float) -> "LogitsProcessor":
        return cls(ctx, seed, SamplingParams(temperature, top_p, top_k, repetition_penalty))

    @classmethod
    def new(cls, ctx, seed: int, temperature: Optional[float], top_p: Optional[float]) -> "LogitsProcessor":
        """LogitsProcessor::new (sampling.rs:50-61)."""
        t = temperature if temperature is not None and temperature >= 1e-7 else 0.0
        return cls(ctx, seed, SamplingParams(t, top_p if top_p is not None else 1.0, 0, 1.0))

    def set_repetition_penalty(self, penalty: float):
        self.params.repetition_penalty = penalty

    def clear_history(self):
        self.previous_tokens.clear()

    def sample(self, logits) -> int:
        u = sampling_uniform(self.seed, len(self.previous_tokens))
        tok = int(sample_logits(self.ctx, logits, [self.params], [u], [self.previous_tokens])[0])
        self.previous_tokens.append(tok)
        return tok
