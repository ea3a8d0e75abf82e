"""The drop-in yue2_cuda_ar_stack (metal.m:718-874 contract) against the oracle's
Model::hidden CPU branch on config 0."""
import ctypes

import numpy as np
import pytest

from oracle.oracle import norm as onorm
from yue2_rs_b200 import _lib, checkpoint

pytestmark = pytest.mark.gpu


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def test_ar_stack_matches_oracle(c1u_dir, c1u_oracle, c1_prompt):
    c = c1u_oracle.config
    H, D, kv, heads, I = c.hidden_size, c.head_dim, c.num_key_value_heads, c.num_attention_heads, c.intermediate_size
    t = {n: a for n, _, _, a in checkpoint.tensors(c1u_dir)}
    to_f = lambda b: (np.asarray(b).astype(np.uint32) << 16).view(np.float32)
    prompt = c1_prompt[0][:300]
    oc = c1u_oracle.cache(400)
    c1u_oracle.prefill(prompt, oc)
    L = _lib.lib()
    names = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
             "mlp.up_proj", "mlp.down_proj"]
    keep = []
    layers = (_lib.GpuLayer * c.num_hidden_layers)()
    for l in range(c.num_hidden_layers):
        for j, n in enumerate(names):
            w = np.ascontiguousarray(t[f"model.layers.{l}.{n}.weight"])
            keep.append(w)
            rows = {0: heads * D, 1: kv * D, 2: kv * D, 3: H, 4: I, 5: I, 6: H}[j]
            layers[l].weights[j] = _lib.GpuWeight(w.ctypes.data, 7, rows, w.size // rows, 0, 1)
        for j, n in enumerate(["input_layernorm", "self_attn.q_norm", "self_attn.k_norm", "post_attention_layernorm"]):
            g = np.ascontiguousarray(to_f(t[f"model.layers.{l}.{n}.weight"]))
            keep.append(g)
            layers[l].norms[j] = g.ctypes.data
        k, v = oc.read(l)
        keep += [k, v]
        layers[l].key, layers[l].value = k.ctypes.data, v.ctypes.data
    tok, pos = c1_prompt[1][0], len(prompt)
    x = np.ascontiguousarray(to_f(t["model.embed_tokens.weight"][tok * H:(tok + 1) * H]))
    half = D // 2
    freq = (np.float32(1) / np.power(np.float32(c.rope_theta), (np.arange(half) * 2).astype(np.float32) / np.float32(D))).astype(np.float32)
    ang = (np.float32(pos) * freq).astype(np.float32)
    from refmath import round_bf16_np
    cos = round_bf16_np(np.cos(ang).astype(np.float32))
    sin = round_bf16_np(np.sin(ang).astype(np.float32))
    out = np.empty(H, dtype=np.float32)
    shadow = np.empty(c.num_hidden_layers * 2 * kv * D, dtype=np.float32)
    ok = L.yue2_cuda_ar_stack(_p(x), _p(out), _p(shadow), ctypes.cast(layers, ctypes.c_void_p), c.num_hidden_layers,
                              H, heads, kv, D, I, pos, 400, 4242, c.rms_norm_eps, _p(cos), _p(sin))
    assert ok == 1, _lib.last_error()
    want = c1u_oracle.hidden([tok], oc)[0]
    got = onorm(to_f(t["model.norm.weight"]), c.rms_norm_eps, out)[0]
    # unit-gain hidden states: within the bf16 reordering noise (about 1% relative here)
    rel = np.linalg.norm(got.astype(np.float64) - want) / np.linalg.norm(want)
    assert rel <= 0.03, rel
    for l in range(c.num_hidden_layers):
        k, v = oc.read(l)
        sk = shadow[l * 2 * kv * D: l * 2 * kv * D + kv * D]
        sv = shadow[l * 2 * kv * D + kv * D: (l + 1) * 2 * kv * D]
        assert np.mean(sk == k[pos]) > 0.9 and np.mean(sv == v[pos]) > 0.9
    L.yue2_cuda_release_cache(4242)
    L.yue2_cuda_release_model()
