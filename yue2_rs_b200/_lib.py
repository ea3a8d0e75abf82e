"""ctypes binding of libyue2cuda.so (include/yue2_cuda.h).

The library is loaded from this package directory only; there is no fallback. A
missing or unloadable library raises ImportError-like RuntimeError on first use.
"""
import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libyue2cuda.so")

c_u64 = ctypes.c_uint64
c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_f = ctypes.c_float
c_p = ctypes.c_void_p
c_size = ctypes.c_size_t

YUE2_OK = 0
ERRORS = {
    -1: "INVALID", -2: "CUDA", -3: "OOM", -4: "CAPACITY", -5: "LOGITS", -6: "EMPTY", -7: "TIMEOUT",
    -8: "VOCAB", -9: "TOKEN",
}


class Yue2Error(RuntimeError):
    """A negative status from the library; `.code` holds it, the message is the reason."""

    def __init__(self, code, message):
        super().__init__(f"{message} (YUE2_ERR_{ERRORS.get(code, code)})")
        self.code = code
        self.message = message


class Config(ctypes.Structure):
    _fields_ = [
        ("hidden_size", c_u64), ("num_hidden_layers", c_u64), ("num_attention_heads", c_u64),
        ("num_key_value_heads", c_u64), ("head_dim", c_u64), ("intermediate_size", c_u64),
        ("vocab_size", c_u64), ("max_position_embeddings", c_u64), ("rms_norm_eps", c_f),
        ("rope_theta", c_f), ("tie_word_embeddings", ctypes.c_int32),
    ]


class CSampling(ctypes.Structure):
    _fields_ = [
        ("temperature", c_f), ("top_p", c_f), ("top_k", c_u64), ("repetition_penalty", c_f),
        ("penalty_window", c_u64), ("min_tokens", c_u64), ("max_tokens", c_u64),
    ]


class CRequest(ctypes.Structure):
    _fields_ = [
        ("prefix", ctypes.POINTER(c_i64)), ("prefix_len", c_u64), ("negative", ctypes.POINTER(c_i64)),
        ("negative_len", c_u64), ("seed", c_u64), ("scale", c_f), ("legacy", ctypes.c_int32),
        ("context_fill", c_u64), ("tokens", ctypes.POINTER(c_i64)), ("count", c_u64), ("truncated", ctypes.c_int32),
        ("status", ctypes.c_int32),
    ]


class CTiming(ctypes.Structure):
    _fields_ = [("seconds", ctypes.c_double), ("prefill_seconds", ctypes.c_double), ("decode_ms", ctypes.c_double),
                ("decode_steps", c_u64), ("kernels_per_step", c_u64)]


class GpuWeight(ctypes.Structure):  # tensor.rs:221-230
    _fields_ = [("raw", c_p), ("mapping", c_size), ("rows", c_size), ("cols", c_size), ("dtype", ctypes.c_int32),
                ("rounded", ctypes.c_int32)]


class GpuLayer(ctypes.Structure):  # tensor.rs:231-237
    _fields_ = [("weights", GpuWeight * 7), ("norms", c_p * 4), ("key", c_p), ("value", c_p)]


_PROTOS = {
    "yue2_last_error": (ctypes.c_char_p, []),
    "yue2_cuda_available": (c_int, []),
    "yue2_cuda_vector_default": (c_int, []),
    "yue2_cuda_name": (ctypes.c_char_p, []),
    "yue2_cuda_vector": (c_int, [c_p, c_p, c_size, c_int, c_int, c_int, c_p, c_size, c_size]),
    "yue2_cuda_clear_weights": (None, []),
    "yue2_cuda_release_model": (None, []),
    "yue2_cuda_release_cache": (None, [c_size]),
    "yue2_cuda_ar_stack": (c_int, [c_p, c_p, c_p, c_p, c_size, c_size, c_size, c_size, c_size, c_size, c_size,
                                   c_size, c_size, c_f, c_p, c_p]),
    "yue2_cuda_cached_attention": (c_int, [c_p, c_p, c_p, c_p, c_size, c_size, c_size, c_size, c_size, c_size]),
    "yue2_cuda_stack": (c_int, [c_p, c_p, c_p, c_size, c_size, c_size, c_size, c_size, c_size, c_size, c_size,
                                c_size, c_f, c_p, c_p]),
    "yue2_cuda_linear": (c_int, [c_p, c_p, c_size, c_int, c_int, c_p, c_size, c_size, c_size]),
    "yue2_cuda_gemm": (c_int, [c_p, c_p, c_p, c_size, c_size, c_size, c_int, c_size, c_size, c_size, c_f]),
    "yue2_cuda_attention": (c_int, [c_p, c_p, c_p, c_p, c_size, c_size, c_size, c_size, c_size, ctypes.c_int64, c_f]),
    "yue2_attention_noalloc": (c_int, [c_p, c_p, c_p, c_p, c_u64, c_u64, c_u64, c_u64, c_p]),
    "yue2_model_create": (c_int, [c_int, ctypes.POINTER(Config), ctypes.POINTER(c_p)]),
    "yue2_model_create_tp": (c_int, [c_int, ctypes.POINTER(Config), c_u64, c_u64, ctypes.POINTER(c_p)]),
    "yue2_tp_export": (c_int, [c_p, c_p]),
    "yue2_tp_connect": (c_int, [c_p, c_p]),
    "yue2_model_set_tensor": (c_int, [c_p, ctypes.c_char_p, c_int, c_p, c_u64, c_u64]),
    "yue2_model_init_synthetic": (c_int, [c_p, c_u64, c_f, c_f]),
    "yue2_model_finalize": (c_int, [c_p]),
    "yue2_model_load_checkpoint": (c_int, [c_p, ctypes.c_char_p, ctypes.POINTER(c_u64)]),
    "yue2_model_enable_nar": (c_int, [c_p, c_u64, c_u64, c_f]),
    "yue2_checkpoint_scan": (c_int, [ctypes.c_char_p, ctypes.POINTER(c_u64)]),
    "yue2_bench_gemm": (c_int, [c_p, c_p, c_p, c_p, c_int, c_int, c_int, c_int, c_int, ctypes.POINTER(ctypes.c_double)]),
    "yue2_model_get_tensor": (c_int, [c_p, ctypes.c_char_p, c_p, c_u64]),
    "yue2_model_free": (None, [c_p]),
    "yue2_cache_create": (c_int, [c_p, c_u64, ctypes.POINTER(c_p)]),
    "yue2_cache_free": (None, [c_p]),
    "yue2_cache_length": (c_int, [c_p, ctypes.POINTER(c_u64)]),
    "yue2_cache_fill_normal": (c_int, [c_p, c_u64, c_u64]),
    "yue2_cache_read": (c_int, [c_p, c_u64, c_u64, c_u64, c_p, c_p]),
    "yue2_forward": (c_int, [c_p, c_p, c_p, c_u64, c_int, c_p]),
    "yue2_prefill": (c_int, [c_p, c_p, c_p, c_u64, c_int, c_p]),
    "yue2_velocity": (c_int, [c_p, c_p, c_p, c_u64, ctypes.c_double, c_p]),
    "yue2_synthesize": (c_int, [c_p, c_p, c_u64, c_p, c_u64, c_u64, c_u64, c_p]),
    "yue2_noise": (c_int, [c_u64, c_u64, c_u64, c_p]),
    "yue2_rng_create": (c_int, [c_p, c_u64, ctypes.POINTER(c_p)]),
    "yue2_rng_free": (None, [c_p]),
    "yue2_rng_state": (c_int, [c_p, c_p, ctypes.POINTER(c_u64)]),
    "yue2_choose": (c_int, [c_p, c_p, c_u64, ctypes.POINTER(CSampling), c_p, c_u64, c_u64, c_int, c_int, c_p,
                            ctypes.POINTER(c_i64)]),
    "yue2_generate": (c_int, [c_p, ctypes.POINTER(CSampling), c_int, ctypes.POINTER(CRequest), c_u64,
                              ctypes.POINTER(CTiming)]),
    "yue2_session_create": (c_int, [c_p, ctypes.POINTER(CSampling), c_int, ctypes.POINTER(CRequest), c_u64,
                                    ctypes.POINTER(c_p)]),
    "yue2_session_step": (c_int, [c_p, c_u64, ctypes.POINTER(c_u64)]),
    "yue2_session_sync": (c_int, [c_p]),
    "yue2_session_collect": (c_int, [c_p, ctypes.POINTER(CRequest)]),
    "yue2_session_stream": (c_p, [c_p]),
    "yue2_session_kernels_per_step": (c_u64, [c_p]),
    "yue2_session_free": (None, [c_p]),
    "yue2_bench_gemv": (c_int, [c_p, c_int, c_int, c_int, ctypes.POINTER(ctypes.c_double),
                                ctypes.POINTER(ctypes.c_double)]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library (loaded once)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(f"{LIB_PATH} is missing: run `python -m yue2_rs_b200.build` (there is no CPU fallback)")
            L = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _PROTOS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def exported_symbols():
    return sorted(_PROTOS)


def check(code):
    """Raise Yue2Error for a negative status; return the status otherwise."""
    if code < 0:
        raise Yue2Error(code, lib().yue2_last_error().decode(errors="replace"))
    return code


def last_error():
    return lib().yue2_last_error().decode(errors="replace")
