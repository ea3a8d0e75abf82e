"""Host-side logic that needs no GPU: configuration checks, checkpoint IO, the library ABI."""
import ctypes
import os
import re

import numpy as np
import pytest

from yue2_rs_b200 import _lib, checkpoint, synth
from yue2_rs_b200.model import Config
from yue2_rs_b200.protocol import Sampling

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    text = open(os.path.join(ROOT, "include", "yue2_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(yue2_\w+)\s*\(", text)))


def test_library_exports_every_declared_entry_point():
    names = header_functions()
    assert len(names) >= 30
    L = ctypes.CDLL(_lib.LIB_PATH)  # loads without a GPU
    for n in names:
        assert hasattr(L, n), n
    assert sorted(_lib.exported_symbols()) == names


def test_no_device_is_an_error_not_a_fallback():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    assert _lib.lib().yue2_cuda_available() == 0
    from yue2_rs_b200 import Model, Yue2Error
    with pytest.raises(Yue2Error):
        Model(synth.config_c1())


def test_sampling_validation_mirrors_protocol():
    Sampling().validate()
    Sampling.abc().validate()
    for bad in (dict(temperature=-0.1), dict(temperature=5.5), dict(top_p=0.0), dict(top_p=1.5), dict(top_k=0),
                dict(repetition_penalty=0.0), dict(penalty_window=0), dict(penalty_window=101),
                dict(min_tokens=10, max_tokens=5), dict(max_tokens=0), dict(temperature=float("nan"))):
        with pytest.raises(ValueError):
            Sampling(**bad).validate()


def test_config_validation(tmp_path):
    c = synth.config_c1()
    c.validate()
    with pytest.raises(ValueError):
        Config(num_attention_heads=6, num_key_value_heads=4).validate()
    p = tmp_path / "config.json"
    p.write_text('{"model_type": "other"}')
    with pytest.raises(ValueError):
        Config.read(str(p))


def test_checkpoint_roundtrip(tmp_path):
    a = np.arange(12, dtype=np.uint16).reshape(3, 4)
    b = np.linspace(0, 1, 5).astype(np.float32)
    checkpoint.write(str(tmp_path / "model.safetensors"), {"a": ("BF16", (3, 4), a), "b": ("F32", (5,), b)})
    got = {n: (code, shape, arr) for n, code, shape, arr in checkpoint.tensors(str(tmp_path))}
    assert got["a"][0] == 0 and got["a"][1] == (3, 4) and (got["a"][2] == a.ravel()).all()
    assert got["b"][0] == 1 and (got["b"][2] == b).all()


def test_synthetic_checkpoint_is_deterministic():
    c = Config(hidden_size=16, num_hidden_layers=1, num_attention_heads=2, num_key_value_heads=1, head_dim=8,
               intermediate_size=32, vocab_size=40, max_latent_frames=4, latent_dim=4)
    a = {n: b for n, _, b in synth.generate(c, 0, norm_mean=1.0)}
    b = {n: b for n, _, b in synth.generate(c, 0, norm_mean=1.0)}
    assert a.keys() == b.keys() and all((a[k] == b[k]).all() for k in a)
    assert "model.layers.0.nar_mlp.down_proj.weight" in a and "latent_pos_embed.pe" in a
    g = a["model.layers.0.input_layernorm.weight"].astype(np.uint32) << 16
    assert np.allclose(g.view(np.float32), 1.0, atol=0.1)


def test_noalloc_attention_rejects_overflowing_shapes_before_any_launch():
    """Shape values whose products would wrap 64 bits are refused up front (no device
    call is made, so this runs without a GPU)."""
    L = _lib.lib()
    p = 256  # aligned, never dereferenced: the shape check comes first
    kv = (1 << 62) + 1
    for heads, kvh in ((2 * kv, kv), (1 << 40, 1), (4, 70000)):
        assert L.yue2_attention_noalloc(p, p, p, p, 64, heads, kvh, 128, None) == -1
        assert "invalid attention shape" in _lib.last_error()
