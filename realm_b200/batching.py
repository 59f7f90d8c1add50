"""Continuous batching: the reference's batching API over the native library.

* ``BatchedRequest``, ``ContinuousBatcher`` and ``BatchStats`` mirror
  crates/realm-runtime/src/batching.rs:10-210. The queue, its locking and its
  rules live in librealm_b200.so (``rb_batcher_*``); this module marshals.
* ``prepare_batch`` mirrors crates/realm-runtime/src/batch_forward.rs:164-189
  (right-padding with token 0 and a validity mask). The device path itself
  needs no padding: ``rb_forward`` takes ragged rows over the paged cache.
* ``Scheduler`` is the continuous-batching decode loop on one ``Model``
  (``rb_scheduler_*``): requests join and leave between steps, and every step
  is one batched ``rb_forward`` over the live requests' rows.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import RealmError, _check, _lib, _sig

_vp, _u32, _i32, _u64 = C.c_void_p, C.c_uint32, C.c_int32, C.c_uint64
_U32P = C.POINTER(C.c_uint32)

NO_EOS = 0xFFFFFFFF
FINISH_NONE, FINISH_MAX_TOKENS, FINISH_EOS, FINISH_LENGTH, FINISH_CANCELLED = range(5)
FINISH_NAMES = {FINISH_NONE: None, FINISH_MAX_TOKENS: "max_tokens", FINISH_EOS: "eos",
                FINISH_LENGTH: "length", FINISH_CANCELLED: "cancelled"}


class _RequestView(C.Structure):
    _fields_ = [("request_id", C.c_uint64), ("prompt_tokens", _U32P), ("n_prompt", C.c_uint32),
                ("n_generated", C.c_uint32), ("generated_tokens", _U32P), ("prompt_text", C.c_char_p),
                ("max_tokens", C.c_uint32), ("is_complete", C.c_uint32)]


class _BatchStats(C.Structure):
    _fields_ = [("total_requests", C.c_uint64), ("active_requests", C.c_uint64),
                ("average_sequence_length", C.c_uint64)]


class _SchedConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("max_batch_size", "max_seq_len", "prefill_chunk", "eos_token",
                                          "tenant_base")]


class _StepEvent(C.Structure):
    _fields_ = [("request_id", C.c_uint64), ("token", C.c_uint32), ("index", C.c_uint32), ("finish", C.c_int32)]


class _SchedStats(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("steps", "rows", "prefill_rows", "decode_rows", "tokens_generated")] + [
        ("queued", C.c_uint32), ("live", C.c_uint32), ("finished", C.c_uint32), ("device_ms", C.c_float)]


_sig("rb_batcher_create", [_u32, _u32, C.POINTER(_vp)])
_sig("rb_batcher_destroy", [_vp])
_sig("rb_batcher_add_request", [_vp, _u64, _vp, _u32, C.c_char_p, _u32])
_sig("rb_batcher_get_batch", [_vp, C.POINTER(_vp)])
_sig("rb_request_list_get", [_vp, _u32, C.POINTER(_RequestView)])
_sig("rb_request_list_free", [_vp])
_sig("rb_batcher_update_request", [_vp, _u64, _u32])
_sig("rb_batcher_remove_request", [_vp, _u64])
_sig("rb_batcher_active_count", [_vp])
_sig("rb_batcher_stats", [_vp, C.POINTER(_BatchStats)])
_sig("rb_model_get_config", [_vp, _i32, _vp])
_sig("rb_ctx_max_rows", [_vp])
_sig("rb_scheduler_create", [_vp, _i32, C.POINTER(_SchedConfig), C.POINTER(_vp)])
_sig("rb_scheduler_destroy", [_vp])
_sig("rb_scheduler_submit", [_vp, _u64, _vp, _u32, _u32])
_sig("rb_scheduler_step", [_vp, C.POINTER(_StepEvent), _u32, _vp])
_sig("rb_scheduler_result", [_vp, _u64, _vp, _u32, C.POINTER(C.c_int32)])
_sig("rb_scheduler_submit_sampled", [_vp, _u64, _vp, _u32, _u32, _vp, _u64])
_sig("rb_scheduler_cancel", [_vp, _u64])
_sig("rb_scheduler_release", [_vp, _u64])
_sig("rb_scheduler_stats", [_vp, C.POINTER(_SchedStats)])


def _u32_array(tokens: Sequence[int]) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64))
    if a.size and (a.min() < 0 or a.max() > 0xFFFFFFFF):
        raise ValueError("token ids must fit in u32")
    return a.astype(np.uint32)


@dataclass
class BatchedRequest:
    """BatchedRequest (batching.rs:10-73)."""
    request_id: int
    prompt_tokens: List[int]
    max_tokens: int
    prompt_text: Optional[str] = None
    generated_tokens: List[int] = field(default_factory=list)
    is_complete: bool = False

    @classmethod
    def new(cls, request_id: int, prompt_tokens: Sequence[int], max_tokens: int) -> "BatchedRequest":
        return cls(request_id, list(prompt_tokens), max_tokens)

    @classmethod
    def with_prompt_text(cls, request_id: int, prompt_tokens: Sequence[int], prompt_text: str,
                         max_tokens: int) -> "BatchedRequest":
        return cls(request_id, list(prompt_tokens), max_tokens, prompt_text)

    def current_seq_len(self) -> int:
        return len(self.prompt_tokens) + len(self.generated_tokens)

    def all_tokens(self) -> List[int]:
        return list(self.prompt_tokens) + list(self.generated_tokens)


@dataclass
class BatchStats:
    """BatchStats (batching.rs:213-219)."""
    total_requests: int
    active_requests: int
    average_sequence_length: int


class ContinuousBatcher:
    """ContinuousBatcher (batching.rs:76-210) backed by rb_batcher_*.

    Errors raise RealmError, whose message is the reference's
    ("Batch queue is full", "Request <id> not found").
    """

    def __init__(self, max_batch_size: int, max_seq_len: int):
        h = _vp()
        _check(_lib.rb_batcher_create(max_batch_size, max_seq_len, C.byref(h)))
        self._h = h
        self.max_batch_size, self.max_seq_len = max_batch_size, max_seq_len

    def __del__(self):
        if getattr(self, "_h", None):
            _lib.rb_batcher_destroy(self._h)
            self._h = None

    def add_request(self, request: BatchedRequest) -> None:
        toks = _u32_array(request.prompt_tokens)
        text = request.prompt_text.encode() if request.prompt_text is not None else None
        _check(_lib.rb_batcher_add_request(self._h, request.request_id, toks.ctypes.data, toks.size, text,
                                           request.max_tokens))
        # a request queued again after some steps keeps the tokens it generated
        for t in request.generated_tokens:
            _check(_lib.rb_batcher_update_request(self._h, request.request_id, int(t)))

    def get_batch(self) -> List[BatchedRequest]:
        lst = _vp()
        n = _check(_lib.rb_batcher_get_batch(self._h, C.byref(lst)))
        out = []
        try:
            v = _RequestView()
            for i in range(n):
                _check(_lib.rb_request_list_get(lst, i, C.byref(v)))
                out.append(BatchedRequest(
                    request_id=int(v.request_id),
                    prompt_tokens=[int(v.prompt_tokens[j]) for j in range(v.n_prompt)],
                    max_tokens=int(v.max_tokens),
                    prompt_text=v.prompt_text.decode() if v.prompt_text is not None else None,
                    generated_tokens=[int(v.generated_tokens[j]) for j in range(v.n_generated)],
                    is_complete=bool(v.is_complete)))
        finally:
            _lib.rb_request_list_free(lst)
        return out

    def update_request(self, request_id: int, new_token: int) -> None:
        _check(_lib.rb_batcher_update_request(self._h, request_id, new_token))

    def remove_request(self, request_id: int) -> None:
        _check(_lib.rb_batcher_remove_request(self._h, request_id))

    def active_count(self) -> int:
        return _check(_lib.rb_batcher_active_count(self._h))

    def stats(self) -> BatchStats:
        s = _BatchStats()
        _check(_lib.rb_batcher_stats(self._h, C.byref(s)))
        return BatchStats(int(s.total_requests), int(s.active_requests), int(s.average_sequence_length))


def prepare_batch(batch_tokens: Sequence[Sequence[int]], max_seq_len: int):
    """prepare_batch (batch_forward.rs:164-189): pad each sequence with 0 up to
    max_seq_len (never truncating) and give a mask that is True on real tokens."""
    padded, masks = [], []
    for toks in batch_tokens:
        pad = max(0, max_seq_len - len(toks))
        padded.append(list(toks) + [0] * pad)
        masks.append([True] * len(toks) + [False] * pad)
    return padded, masks


@dataclass
class StepEvent:
    request_id: int
    token: int
    index: int
    finish: Optional[str]


class Scheduler:
    """Continuous-batching decode scheduler on one realm_b200.Model.

    submit() queues a request; step() admits queued requests into free slots,
    runs one batched forward over the live ones (decode rows first, then
    prompt chunks) and returns the tokens it generated as StepEvents, with
    their logits rows when want_logits. run() steps until everything
    submitted has finished and returns each request's generated tokens.
    """

    def __init__(self, model, max_batch_size: int, max_seq_len: int = 0, prefill_chunk: int = 0,
                 eos_token: Optional[int] = None, tenant_base: int = 0):
        self.model = model
        cfg = _SchedConfig(max_batch_size, max_seq_len, prefill_chunk, NO_EOS if eos_token is None else eos_token,
                           tenant_base)
        h = _vp()
        _check(_lib.rb_scheduler_create(model.ctx.handle, model.handle, C.byref(cfg), C.byref(h)))
        self._h = h
        self.max_batch_size = max_batch_size
        self.vocab = int(model.cfg["vocab"])
        self._ev = (_StepEvent * max_batch_size)()
        self._logits = None

    def close(self):
        if getattr(self, "_h", None):
            h, self._h = self._h, None
            _check(_lib.rb_scheduler_destroy(h))

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, request_id: int, prompt: Sequence[int], max_tokens: int, sampling=None, seed: int = 0) -> None:
        """sampling: a realm_b200.SamplingParams (None: greedy); seed: its uniform stream."""
        toks = _u32_array(prompt)
        if sampling is None:
            _check(_lib.rb_scheduler_submit(self._h, request_id, toks.ctypes.data if toks.size else None, toks.size,
                                            max_tokens))
            return
        p = sampling.c()
        _check(_lib.rb_scheduler_submit_sampled(self._h, request_id, toks.ctypes.data if toks.size else None,
                                                toks.size, max_tokens, C.byref(p), seed & (2**64 - 1)))

    def step(self, want_logits: bool = False):
        """One step. Returns [StepEvent], or ([StepEvent], logits [n][vocab]) with want_logits."""
        lg = None
        if want_logits:
            if self._logits is None:
                self._logits = np.empty((self.max_batch_size, self.vocab), np.float32)
            lg = self._logits
        n = _check(_lib.rb_scheduler_step(self._h, self._ev, self.max_batch_size,
                                          lg.ctypes.data if lg is not None else None))
        ev = [StepEvent(int(e.request_id), int(e.token), int(e.index), FINISH_NAMES[e.finish])
              for e in self._ev[:n]]
        return (ev, lg[:n].copy()) if want_logits else ev

    def result(self, request_id: int):
        """(generated tokens, finish reason or None while running)."""
        fin = C.c_int32()
        n = _check(_lib.rb_scheduler_result(self._h, request_id, None, 0, C.byref(fin)))
        out = np.empty(n, np.uint32)
        if n:
            _check(_lib.rb_scheduler_result(self._h, request_id, out.ctypes.data, n, C.byref(fin)))
        return [int(t) for t in out], FINISH_NAMES[fin.value]

    def cancel(self, request_id: int) -> None:
        _check(_lib.rb_scheduler_cancel(self._h, request_id))

    def release(self, request_id: int) -> None:
        _check(_lib.rb_scheduler_release(self._h, request_id))

    def stats(self) -> Dict[str, float]:
        s = _SchedStats()
        _check(_lib.rb_scheduler_stats(self._h, C.byref(s)))
        return {n: getattr(s, n) for n, _ in _SchedStats._fields_}

    def run(self, max_steps: int = 1 << 30) -> Dict[int, List[int]]:
        """Steps until nothing is queued or live; returns {request_id: tokens} of the events seen."""
        out: Dict[int, List[int]] = {}
        for _ in range(max_steps):
            before = self.stats()
            if before["queued"] == 0 and before["live"] == 0:
                break
            ev = self.step()
            if self.stats()["steps"] == before["steps"]:
                raise RealmError(-21, "scheduler made no progress (queued requests do not fit the KV pool)")
            for e in ev:
                out.setdefault(e.request_id, []).append(e.token)
        return out
