"""ctypes binding of the CPU checker (liboracle.so) -- TEST INFRASTRUCTURE.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module.
It restates the reference's CPU decode math (see yue2_oracle.cpp's header).
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")

c_u64, c_i64, c_p, c_f, c_int = ctypes.c_uint64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_float, ctypes.c_int


class OrcSampling(ctypes.Structure):
    _fields_ = [("temperature", c_f), ("top_p", c_f), ("top_k", c_u64), ("repetition_penalty", c_f),
                ("penalty_window", c_u64), ("min_tokens", c_u64), ("max_tokens", c_u64)]


_P = {
    "orc_last_error": (ctypes.c_char_p, []),
    "orc_set_threads": (None, [c_int]),
    "orc_set_dot_order": (None, [c_int]),
    "orc_max_threads": (c_int, []),
    "orc_model_create": (c_p, [c_p, c_p]),
    "orc_model_free": (None, [c_p]),
    "orc_model_set": (c_int, [c_p, ctypes.c_char_p, c_int, c_p, c_u64, c_u64]),
    "orc_model_finalize": (c_int, [c_p]),
    "orc_model_init_synthetic": (c_int, [c_p, c_u64, c_f, c_f]),
    "orc_cache_create": (c_p, [c_p, c_u64]),
    "orc_cache_free": (None, [c_p]),
    "orc_cache_length": (c_u64, [c_p]),
    "orc_cache_read": (c_int, [c_p, c_u64, c_p, c_p]),
    "orc_cache_write": (c_int, [c_p, c_p, c_u64, c_p]),
    "orc_hidden": (c_int, [c_p, c_p, c_p, c_u64, c_p]),
    "orc_forward": (c_int, [c_p, c_p, c_p, c_u64, c_int, c_p]),
    "orc_prefill": (c_int, [c_p, c_p, c_p, c_u64, c_int, c_p]),
    "orc_attention": (c_int, [c_p, c_p, c_p, c_p, c_u64, c_u64, c_u64, c_u64]),
    "orc_linear": (c_int, [c_p, c_u64, c_u64, c_p, c_u64, c_p]),
    "orc_norm": (c_int, [c_p, c_u64, c_f, c_p, c_u64, c_p]),
    "orc_rng_create": (c_p, [c_u64]),
    "orc_rng_free": (None, [c_p]),
    "orc_rng_next_u32": (ctypes.c_uint32, [c_p]),
    "orc_rng_uniform_f64": (ctypes.c_double, [c_p]),
    "orc_rng_uniform_f32": (c_f, [c_p]),
    "orc_rng_discard": (None, [c_p, c_u64]),
    "orc_rng_state": (None, [c_p, c_p, ctypes.POINTER(c_u64)]),
    "orc_sampling_validate": (c_int, [ctypes.POINTER(OrcSampling)]),
    "orc_choose": (c_int, [c_p, c_u64, ctypes.POINTER(OrcSampling), c_p, c_u64, c_u64, c_int, c_int, c_p,
                           ctypes.POINTER(c_i64)]),
    "orc_cfg_mix": (None, [c_p, c_p, c_f, c_p, c_u64]),
    "orc_det_expf": (c_f, [c_f]),
    "orc_det_log1p": (ctypes.c_double, [ctypes.c_double]),
    "orc_round_bf16": (c_f, [c_f]),
    "orc_powi": (c_f, [c_f, c_int]),
    "orc_generate": (c_int, [c_p, c_p, c_u64, c_p, c_u64, ctypes.POINTER(OrcSampling), c_u64, c_int, c_f, c_int,
                             c_p, ctypes.POINTER(c_u64), ctypes.POINTER(c_int)]),
    "orc_model_nar": (c_int, [c_p, c_u64, c_u64, c_f]),
    "orc_velocity": (c_int, [c_p, c_p, c_p, c_u64, ctypes.c_double, c_p]),
    "orc_normal_tensor": (c_int, [c_u64, c_u64, c_u64, c_p]),
    "orc_synthesize": (c_int, [c_p, c_p, c_u64, c_p, c_u64, c_u64, c_u64, c_p]),
}

_lib = None


def build():
    subprocess.check_call(["make", "-s", "-C", HERE])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        for k, (r, a) in _P.items():
            f = getattr(L, k)
            f.restype, f.argtypes = r, a
        _lib = L
    return _lib


class OracleError(RuntimeError):
    pass


def _ck(rc):
    if rc < 0:
        raise OracleError(lib().orc_last_error().decode())
    return rc


def _ptr(a):
    return a.ctypes.data_as(c_p)


def sampling_c(s):
    return OrcSampling(s.temperature, s.top_p, s.top_k, s.repetition_penalty, s.penalty_window, s.min_tokens,
                       s.max_tokens)


def set_threads(n):
    lib().orc_set_threads(n)


def set_dot_order(order):
    """0: 16 interleaved partial sums (default); 1: strictly sequential dot products."""
    lib().orc_set_dot_order(order)


class OracleModel:
    def __init__(self, config):
        self.config = c = config
        cfg = np.array([c.hidden_size, c.num_hidden_layers, c.num_attention_heads, c.num_key_value_heads,
                        c.head_dim, c.intermediate_size, c.vocab_size, c.max_position_embeddings,
                        int(bool(c.tie_word_embeddings))], dtype=np.uint64)
        f = np.array([c.rms_norm_eps, c.rope_theta], dtype=np.float32)
        self._h = lib().orc_model_create(_ptr(cfg), _ptr(f))
        if not self._h:
            raise OracleError(lib().orc_last_error().decode())

    @classmethod
    def from_tensors(cls, config, items, nar=False):
        """items: iterable of (name, dtype code, shape, array). nar: also keep the NAR
        pathway's tensors (Model::velocity)."""
        m = cls(config)
        if nar:
            _ck(lib().orc_model_nar(m._h, config.latent_dim, config.max_latent_frames, config.timestep_shift))
        for name, code, shape, arr in items:
            rows, cols = (shape[0], int(np.prod(shape[1:]))) if len(shape) > 1 else (1, shape[0])
            m.set(name, arr, code, rows, cols)
        _ck(lib().orc_model_finalize(m._h))
        return m

    @classmethod
    def synthetic(cls, config, seed, std=0.02, norm_mean=0.0, nar=False):
        """Seeded synthetic weights (nar: the NAR tensors too), for timing."""
        m = cls(config)
        if nar:
            _ck(lib().orc_model_nar(m._h, config.latent_dim, config.max_latent_frames, config.timestep_shift))
        _ck(lib().orc_model_init_synthetic(m._h, seed, std, norm_mean))
        return m

    def set(self, name, arr, code, rows, cols):
        arr = np.ascontiguousarray(arr)
        return _ck(lib().orc_model_set(self._h, name.encode(), code, _ptr(arr), rows, cols))

    def finalize(self):
        _ck(lib().orc_model_finalize(self._h))

    def close(self):
        if self._h:
            lib().orc_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def cache(self, capacity):
        return OracleCache(self, capacity)

    def forward(self, ids, cache, phase=2):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        out = np.empty(self.config.vocab_size, dtype=np.float32)
        _ck(lib().orc_forward(self._h, cache._h, _ptr(ids), ids.size, phase, _ptr(out)))
        return out

    def prefill(self, ids, cache, phase=2, logits=True):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        out = np.empty(self.config.vocab_size, dtype=np.float32) if logits else None
        _ck(lib().orc_prefill(self._h, cache._h, _ptr(ids), ids.size, phase, _ptr(out) if logits else None))
        return out

    def velocity(self, state, cache, raw_t):
        """Model::velocity (src/model.rs:611-697) with nar_cond_end = 0: state [rows, latent]
        (bf16-valued f32) -> velocity [rows, latent]. The cache is not changed."""
        st = np.ascontiguousarray(state, dtype=np.float32)
        out = np.empty_like(st)
        _ck(lib().orc_velocity(self._h, cache._h, _ptr(st), st.shape[0], float(raw_t), _ptr(out)))
        return out

    def synthesize(self, prefix, codec, seed, steps):
        """Model::synthesize (src/model.rs:699-776): latents [len(codec), 64]."""
        p = np.ascontiguousarray(prefix, dtype=np.int64)
        c = np.ascontiguousarray(codec, dtype=np.int64)
        out = np.empty((c.size, 64), dtype=np.float32)
        _ck(lib().orc_synthesize(self._h, _ptr(p), p.size, _ptr(c), c.size, seed, steps, _ptr(out)))
        return out

    def hidden(self, ids, cache):
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        out = np.empty((ids.size, self.config.hidden_size), dtype=np.float32)
        _ck(lib().orc_hidden(self._h, cache._h, _ptr(ids), ids.size, _ptr(out)))
        return out

    def generate(self, prefix, sampling, seed, phase, negative=None, scale=1.0, legacy=False):
        p = np.ascontiguousarray(prefix, dtype=np.int64)
        n = np.ascontiguousarray(negative if negative is not None else [0], dtype=np.int64)
        toks = np.zeros(sampling.max_tokens, dtype=np.int64)
        cnt, trunc = c_u64(), c_int()
        s = sampling_c(sampling)
        _ck(lib().orc_generate(self._h, _ptr(p), p.size, _ptr(n) if negative is not None else None,
                               len(negative) if negative is not None else 0, ctypes.byref(s), seed, phase, scale,
                               int(bool(legacy)), _ptr(toks), ctypes.byref(cnt), ctypes.byref(trunc)))
        return toks[: cnt.value].tolist(), bool(trunc.value)


class OracleCache:
    def __init__(self, model, capacity):
        self.model = model
        self._h = lib().orc_cache_create(model._h, capacity)

    @property
    def length(self):
        return lib().orc_cache_length(self._h)

    def read(self, layer):
        c = self.model.config
        n = self.length
        w = c.num_key_value_heads * c.head_dim
        k = np.empty((n, w), dtype=np.float32)
        v = np.empty((n, w), dtype=np.float32)
        _ck(lib().orc_cache_read(self._h, layer, _ptr(k), _ptr(v)))
        return k, v

    def write(self, length, bits):
        """bits: bf16 uint16 [layers][2][length][kv*dim]."""
        bits = np.ascontiguousarray(bits, dtype=np.uint16)
        _ck(lib().orc_cache_write(self._h, self.model._h, length, _ptr(bits)))

    def close(self):
        if self._h:
            lib().orc_cache_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class OracleRng:
    def __init__(self, seed):
        self._h = lib().orc_rng_create(seed)

    def next_u32(self):
        return lib().orc_rng_next_u32(self._h)

    def uniform_f64(self):
        return lib().orc_rng_uniform_f64(self._h)

    def uniform_f32(self):
        return lib().orc_rng_uniform_f32(self._h)

    def discard(self, n):
        lib().orc_rng_discard(self._h, n)

    def state(self):
        st = np.empty(624, dtype=np.uint32)
        nxt = c_u64()
        lib().orc_rng_state(self._h, _ptr(st), ctypes.byref(nxt))
        return st, nxt.value

    def __del__(self):
        try:
            lib().orc_rng_free(self._h)
        except Exception:
            pass


def normal_tensor(seed, rows, cols):
    """Generator::new(seed).normal_tensor(rows, cols) (src/sampling.rs:63-78)."""
    out = np.empty((rows, cols), dtype=np.float32)
    _ck(lib().orc_normal_tensor(seed, rows, cols, _ptr(out)))
    return out


def choose(logits, sampling, history, step, phase, legacy, rng):
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    hist = np.ascontiguousarray(history, dtype=np.int64)
    out = c_i64()
    s = sampling_c(sampling)
    _ck(lib().orc_choose(_ptr(logits), logits.size, ctypes.byref(s), _ptr(hist) if hist.size else None, hist.size,
                         step, phase, int(bool(legacy)), rng._h, ctypes.byref(out)))
    return out.value


def cfg_mix(c, u, scale):
    c = np.ascontiguousarray(c, dtype=np.float32)
    u = np.ascontiguousarray(u, dtype=np.float32)
    out = np.empty_like(c)
    lib().orc_cfg_mix(_ptr(c), _ptr(u), scale, _ptr(out), c.size)
    return out


def attention(q, k, v, heads, kv, dim):
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    out = np.empty(heads * dim, dtype=np.float32)
    _ck(lib().orc_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), k.shape[0], heads, kv, dim))
    return out


def linear(w_bits, x):
    """Linear::apply + finish: w_bits bf16 [out, in], x f32 [rows, in] -> [rows, out]."""
    w_bits = np.ascontiguousarray(w_bits, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, w_bits.shape[1])
    y = np.empty((x.shape[0], w_bits.shape[0]), dtype=np.float32)
    _ck(lib().orc_linear(_ptr(w_bits), w_bits.shape[0], w_bits.shape[1], _ptr(x), x.shape[0], _ptr(y)))
    return y


def norm(gamma, eps, x):
    gamma = np.ascontiguousarray(gamma, dtype=np.float32)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, gamma.size)
    out = np.empty_like(x)
    _ck(lib().orc_norm(_ptr(gamma), gamma.size, eps, _ptr(x), x.shape[0], _ptr(out)))
    return out
