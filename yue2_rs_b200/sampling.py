"""Request-local MT19937, sampling::choose and sampling::generate on the device
(reference: src/sampling.rs). The decode loop runs as one CUDA-graph launch per token;
the host only enqueues launches and collects the tokens at the end."""
import ctypes
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from .protocol import Phase, Sampling


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


class Generator:
    """Generator (src/sampling.rs:10-62) with its state on the model's device."""

    def __init__(self, model, seed):
        self.model = model
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().yue2_rng_create(model._h, seed, ctypes.byref(h)))
        self._h = h
        model._children.add(self)

    def state(self):
        st = np.empty(624, dtype=np.uint32)
        nxt = ctypes.c_uint64()
        _lib.check(_lib.lib().yue2_rng_state(self._h, _ptr(st), ctypes.byref(nxt)))
        return st, nxt.value

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().yue2_rng_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def choose(model, logits, sampling, history, step, phase, legacy, rng):
    """sampling::choose (src/sampling.rs:103-215) evaluated by the device sampler."""
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    hist = np.ascontiguousarray(history, dtype=np.int64)
    out = ctypes.c_int64()
    s = sampling.to_c()
    _lib.check(_lib.lib().yue2_choose(model._h, _ptr(logits), logits.size, ctypes.byref(s),
                                      _ptr(hist) if hist.size else None, hist.size, step, int(phase),
                                      int(bool(legacy)), rng._h, ctypes.byref(out)))
    return out.value


@dataclass
class Generated:
    """sampling::Generated (src/sampling.rs:216-221)."""

    tokens: list
    truncated: bool
    seconds: float
    prefill_seconds: float
    decode_ms: float = 0.0
    decode_steps: int = 0


@dataclass
class Request:
    prefix: list
    seed: int
    negative: list = None
    scale: float = 1.0
    legacy: bool = False
    context_fill: int = 0  # synthetic N(0,1) KV positions ahead of the prefixes


def _c_requests(requests, max_tokens):
    keep, reqs = [], (_lib.CRequest * len(requests))()
    for i, r in enumerate(requests):
        p = np.ascontiguousarray(r.prefix, dtype=np.int64)
        n = np.ascontiguousarray(r.negative if r.negative is not None else [], dtype=np.int64)
        t = np.zeros(max_tokens, dtype=np.int64)
        keep += [p, n, t]
        reqs[i].prefix = p.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
        reqs[i].prefix_len = p.size
        reqs[i].negative = n.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)) if r.negative is not None else None
        reqs[i].negative_len = n.size
        reqs[i].seed = r.seed
        reqs[i].scale = r.scale
        reqs[i].legacy = int(bool(r.legacy))
        reqs[i].context_fill = int(r.context_fill)
        reqs[i].tokens = t.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
    return reqs, keep


def generate_batch(model, requests, sampling, phase):
    """sampling::generate for several songs at once (all CFG rows in one weight pass)."""
    sampling.validate()
    reqs, keep = _c_requests(requests, sampling.max_tokens)
    timing = _lib.CTiming()
    s = sampling.to_c()
    rc = _lib.lib().yue2_generate(model._h, ctypes.byref(s), int(phase), reqs, len(requests), ctypes.byref(timing))
    _lib.check(rc)
    out = []
    for i in range(len(requests)):
        toks = keep[3 * i + 2][: reqs[i].count].tolist()
        out.append(Generated(toks, bool(reqs[i].truncated), timing.seconds, timing.prefill_seconds,
                             timing.decode_ms, timing.decode_steps))
    return out


def generate(model, prefix, sampling, seed, phase, negative=None, scale=1.0, legacy=False):
    """sampling::generate (src/sampling.rs:222-294)."""
    return generate_batch(model, [Request(prefix, seed, negative, scale, legacy)], sampling, phase)[0]


class Session:
    """The decode loop of generate_batch split at its step boundary (prefill + first draw
    at construction, `step(k)` enqueues k decode steps, `collect()` waits and returns)."""

    def __init__(self, model, requests, sampling, phase):
        sampling.validate()
        self.model, self.sampling, self.n = model, sampling, len(requests)
        self._reqs, self._keep = _c_requests(requests, sampling.max_tokens)
        h = ctypes.c_void_p()
        s = sampling.to_c()
        _lib.check(_lib.lib().yue2_session_create(model._h, ctypes.byref(s), int(phase), self._reqs, self.n,
                                                  ctypes.byref(h)))
        self._h = h
        model._children.add(self)

    @property
    def cuda_stream(self):
        return _lib.lib().yue2_session_stream(self._h)

    @property
    def kernels_per_step(self):
        return _lib.lib().yue2_session_kernels_per_step(self._h)

    def step(self, k):
        n = ctypes.c_uint64()
        _lib.check(_lib.lib().yue2_session_step(self._h, k, ctypes.byref(n)))
        return n.value

    def sync(self):
        _lib.check(_lib.lib().yue2_session_sync(self._h))

    def collect(self):
        _lib.check(_lib.lib().yue2_session_collect(self._h, self._reqs))
        return [(self._keep[3 * i + 2][: self._reqs[i].count].tolist(), bool(self._reqs[i].truncated))
                for i in range(self.n)]

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().yue2_session_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
