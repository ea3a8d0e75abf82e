"""Device model and KV caches: the decode entry points of the reference's src/model.rs
(Model::open/forward/forward_phase/prefill/prefill_phase, Cache) on libyue2cuda."""
import atexit
import ctypes
import json
import math
import os
import weakref
from dataclasses import dataclass

import numpy as np

from . import _lib, checkpoint
from .protocol import CONTEXT, Phase


@dataclass
class Config:
    """model.rs Config (src/model.rs:11-75) with the same defaults and validation."""

    hidden_size: int = 2048
    num_hidden_layers: int = 28
    num_attention_heads: int = 16
    num_key_value_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 6144
    vocab_size: int = 184704
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    max_position_embeddings: int = CONTEXT
    latent_dim: int = 64
    max_latent_frames: int = CONTEXT
    timestep_shift: float = 1.0
    tie_word_embeddings: bool = False

    @classmethod
    def read(cls, path):
        with open(path) as f:
            v = json.load(f)
        if v.get("model_type", "yue2") != "yue2" or v.get("latent_type", "vae") != "vae":
            raise ValueError("Expected YuE2 VAE-latent model")
        c = cls(**{k: v[k] for k in cls.__dataclass_fields__ if k in v})
        c.validate()
        return c

    def validate(self):
        ints = [self.hidden_size, self.num_hidden_layers, self.num_attention_heads, self.num_key_value_heads,
                self.head_dim, self.intermediate_size, self.vocab_size, self.latent_dim, self.max_latent_frames]
        if (0 in ints or self.num_attention_heads % self.num_key_value_heads or self.head_dim % 2
                or not (self.rope_theta > 0 and math.isfinite(self.rope_theta))
                or not (self.rms_norm_eps > 0 and math.isfinite(self.rms_norm_eps))
                or not (self.timestep_shift > 0 and math.isfinite(self.timestep_shift))):
            raise ValueError("Invalid transformer configuration")
        return self

    def to_c(self):
        return _lib.Config(self.hidden_size, self.num_hidden_layers, self.num_attention_heads,
                           self.num_key_value_heads, self.head_dim, self.intermediate_size, self.vocab_size,
                           self.max_position_embeddings, float(self.rms_norm_eps), float(self.rope_theta),
                           int(bool(self.tie_word_embeddings)))

    def json(self):
        d = {k: getattr(self, k) for k in self.__dataclass_fields__}
        d.update(model_type="yue2", latent_type="vae")
        return d


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


_LIVE = weakref.WeakSet()


@atexit.register
def _release_all():
    """Free device objects while the CUDA runtime is still up (module globals would
    otherwise be finalised after it has been torn down)."""
    for m in list(_LIVE):
        try:
            m.close()
        except Exception:
            pass


class Model:
    """A model resident on one GPU. Tensors are uploaded by their checkpoint names."""

    def __init__(self, config, device=0, tp=None):
        """tp = (rank, world): this process's shard of a tensor-parallel model
        (yue2_model_create_tp); connect the ranks with yue2_rs_b200.tp.connect."""
        self.config = config.validate()
        self.device = device
        self.tp = tp
        h = ctypes.c_void_p()
        c = config.to_c()
        if tp is None:
            _lib.check(_lib.lib().yue2_model_create(device, ctypes.byref(c), ctypes.byref(h)))
        else:
            _lib.check(_lib.lib().yue2_model_create_tp(device, ctypes.byref(c), int(tp[0]), int(tp[1]),
                                                       ctypes.byref(h)))
        self._h = h
        self._children = weakref.WeakSet()  # caches/generators to release before the model
        _LIVE.add(self)

    # ---- construction
    @classmethod
    def open(cls, path, device=0, loader="native", nar=False):
        """Model::open (src/model.rs:418-451): config.json + safetensors under `path`. The
        native loader (yue2_model_load_checkpoint) validates the headers and uploads through
        pinned staging; loader="python" reads with numpy and calls set_tensor per tensor.
        nar=True also loads the flow-matching tensors that `velocity` uses."""
        m = cls(Config.read(os.path.join(path, "config.json")), device)
        if nar:
            m.enable_nar()
        if loader == "native":
            _lib.check(_lib.lib().yue2_model_load_checkpoint(m._h, os.fsencode(path), None))
        else:
            for name, code, shape, arr in checkpoint.tensors(path):
                rows, cols = (shape[0], int(np.prod(shape[1:]))) if len(shape) > 1 else (1, shape[0] if shape else 1)
                m.set_tensor(name, arr, code, rows, cols)
        m.finalize()
        return m

    @classmethod
    def synthetic(cls, config, seed, std=0.02, norm_mean=0.0, device=0, nar=False, tp=None):
        """Seeded synthetic weights generated on the device: matrices N(0, std), RMSNorm
        gains norm_mean + N(0, std), bf16. nar=True adds the flow-matching tensors. tp =
        (rank, world): the shard of the same weights that rank holds."""
        m = cls(config, device, tp=tp)
        if nar:
            m.enable_nar()
        _lib.check(_lib.lib().yue2_model_init_synthetic(m._h, seed, std, norm_mean))
        m.finalize()
        return m

    def enable_nar(self):
        """Device slots for the NAR tensors (yue2_model_enable_nar); load them afterwards."""
        c = self.config
        _lib.check(_lib.lib().yue2_model_enable_nar(self._h, c.latent_dim, c.max_latent_frames, c.timestep_shift))
        return self

    def set_tensor(self, name, arr, dtype=None, rows=None, cols=None):
        arr = np.ascontiguousarray(arr)
        if dtype is None:
            dtype = {np.dtype(np.uint16): 0, np.dtype(np.float32): 1, np.dtype(np.float16): 2}[arr.dtype]
        if rows is None:
            rows, cols = (arr.shape[0], int(np.prod(arr.shape[1:]))) if arr.ndim > 1 else (1, arr.size)
        return _lib.check(_lib.lib().yue2_model_set_tensor(self._h, name.encode(), dtype, _ptr(arr), rows, cols))

    def get_tensor(self, name, count):
        out = np.empty(count, dtype=np.uint16)
        _lib.check(_lib.lib().yue2_model_get_tensor(self._h, name.encode(), _ptr(out), count))
        return out

    def finalize(self):
        _lib.check(_lib.lib().yue2_model_finalize(self._h))
        return self

    def close(self):
        if getattr(self, "_h", None):
            for child in list(self._children):
                child.close()
            _lib.lib().yue2_model_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---- decode entry points
    def new_cache(self, capacity):
        return Cache(self, capacity)

    def forward_rows(self, caches, ids, phase=Phase.VOCAB):
        """One new id for each of up to 256 distinct caches in one pass (GEMV for 1-2 rows, GEMMs
        from 3); logits [rows, vocab]."""
        n = len(caches)
        arr = (ctypes.c_void_p * n)(*[c._h for c in caches])
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        out = np.empty((n, self.config.vocab_size), dtype=np.float32)
        _lib.check(_lib.lib().yue2_forward(self._h, arr, _ptr(ids), n, int(phase), _ptr(out)))
        return out

    def forward(self, ids, cache):
        """Model::forward (model.rs:465-468): logits of the last id, full vocabulary."""
        return self.forward_phase(ids, cache, Phase.VOCAB)

    def forward_phase(self, ids, cache, phase):
        """Model::forward_phase (model.rs:469-477)."""
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        if ids.size == 1:
            return self.forward_rows([cache], ids, phase)[0]
        out = np.empty(self.config.vocab_size, dtype=np.float32)
        _lib.check(_lib.lib().yue2_prefill(self._h, cache._h, _ptr(ids), ids.size, int(phase), _ptr(out)))
        return out

    def prefill_phase(self, ids, capacity, phase):
        """Model::prefill_phase (model.rs:508-522) -> (Cache, logits)."""
        cache = Cache(self, capacity)
        return cache, self.forward_phase(ids, cache, phase)

    def prefill(self, ids, capacity, logits=True):
        """Model::prefill (model.rs:592-610) -> (Cache, logits or None)."""
        if len(ids) == 0 or capacity < len(ids):
            raise _lib.Yue2Error(-1, "Invalid prefill/cache capacity")
        cache = Cache(self, capacity)
        ids = np.ascontiguousarray(ids, dtype=np.int64)
        out = np.empty(self.config.vocab_size, dtype=np.float32) if logits else None
        _lib.check(_lib.lib().yue2_prefill(self._h, cache._h, _ptr(ids), ids.size, int(Phase.VOCAB),
                                           _ptr(out) if logits else None))
        return cache, out


    def velocity(self, state, cache, raw_t):
        """Model::velocity (model.rs:611-697, nar_cond_end 0): [rows, latent_dim] f32 velocity
        of the bf16-valued latent frames `state` at logit time `raw_t` over `cache`'s prefix."""
        state = np.ascontiguousarray(state, dtype=np.float32).reshape(-1, self.config.latent_dim)
        out = np.empty_like(state)
        _lib.check(_lib.lib().yue2_velocity(self._h, cache._h, _ptr(state), state.shape[0], float(raw_t),
                                            _ptr(out)))
        return out


    def synthesize(self, prefix, codec, seed, steps=32):
        """Model::synthesize (model.rs:699-776): latents [len(codec), 64] of one song."""
        p = np.ascontiguousarray(prefix, dtype=np.int64)
        c = np.ascontiguousarray(codec, dtype=np.int64)
        out = np.empty((c.size, 64), dtype=np.float32)
        _lib.check(_lib.lib().yue2_synthesize(self._h, _ptr(p), p.size, _ptr(c), c.size, seed, steps, _ptr(out)))
        return out


def noise(seed, rows, cols):
    """Generator::new(seed).normal_tensor(rows, cols) (sampling.rs:63-78), on the host."""
    out = np.empty((rows, cols), dtype=np.float32)
    _lib.check(_lib.lib().yue2_noise(seed, rows, cols, _ptr(out)))
    return out


class Cache:
    """Cache (src/model.rs:276-306): paged bf16 KV on the device, released on drop."""

    def __init__(self, model, capacity):
        self.model = model
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().yue2_cache_create(model._h, capacity, ctypes.byref(h)))
        self._h = h
        self.capacity = capacity
        model._children.add(self)

    @property
    def length(self):
        n = ctypes.c_uint64()
        _lib.check(_lib.lib().yue2_cache_length(self._h, ctypes.byref(n)))
        return n.value

    def fill_normal(self, to, seed):
        _lib.check(_lib.lib().yue2_cache_fill_normal(self._h, to, seed))

    def read(self, layer, begin, count):
        c = self.model.config
        world = self.model.tp[1] if self.model.tp else 1
        w = c.num_key_value_heads // world * c.head_dim  # this rank's KV heads
        k = np.empty((count, w), dtype=np.uint16)
        v = np.empty((count, w), dtype=np.uint16)
        _lib.check(_lib.lib().yue2_cache_read(self._h, layer, begin, count, _ptr(k), _ptr(v)))
        return k, v

    def close(self):
        if getattr(self, "_h", None):
            _lib.lib().yue2_cache_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
