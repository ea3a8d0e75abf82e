"""The oracle's Model::velocity (src/model.rs:611-697, nar_cond_end 0) against an
independent float64 numpy restatement of the same function over the same bf16 tensors.
The reference has no test or golden vector for velocity; its pieces (Linear, Norm, Rotary,
attention) are the ones the AR-path fixtures pin, so this check covers how velocity puts
them together: the zero padding rows, the biased Linears, the timestep embedding, the
position table clamped at max_latent_frames, no causal mask over prefix + latent rows, the
final norm and the row slice. float64 against the oracle's bf16 roundings: a relative
tolerance. Also: the cache is unchanged and the output is bf16-valued.
"""
import math

import numpy as np
import pytest

from oracle import oracle as orc
from yue2_rs_b200 import checkpoint

REL_L2 = 3e-2


def _f(arr, code):
    if code == 0:  # bf16 bits
        return (np.asarray(arr, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    return np.asarray(arr, dtype=np.float64)


@pytest.fixture(scope="module")
def nar(c1u_dir, c1_config):
    items = list(checkpoint.tensors(c1u_dir))
    w = {name: _f(arr, code).reshape(shape) for name, code, shape, arr in items}
    m = orc.OracleModel.from_tensors(c1_config, items, nar=True)
    yield m, w
    m.close()


def _rms(x, g, eps):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * g


def _rope(x, pos, c):
    half = c.head_dim // 2
    freq = 1.0 / np.power(float(c.rope_theta), np.arange(half) * 2.0 / c.head_dim)
    ang = pos[:, None] * freq[None, :]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    left, right = x[..., :half], x[..., half:]
    return np.concatenate([left * cos - right * sin, right * cos + left * sin], -1)


def _velocity(w, c, state, keys, values, length, raw_t):
    """model.rs:611-697 in float64: keys/values are the cache's bf16 prefix per layer."""
    D, H, n = c.latent_dim, c.hidden_size, state.shape[0] + 2
    padded = np.zeros((n, D))
    padded[1:n - 1] = state
    x = padded @ w["vae2llm.weight"].T + w["vae2llm.bias"]
    raw = float(np.float32(raw_t))
    sig = 1.0 / (1.0 + math.exp(-raw))
    t = c.timestep_shift * sig / (1.0 + (c.timestep_shift - 1.0) * sig)
    f = np.exp(-math.log(10000.0) * np.arange(128) / 128.0)
    sinus = np.concatenate([np.cos(t * f), np.sin(t * f)])
    time = sinus @ w["time_embedder.mlp.0.weight"].T + w["time_embedder.mlp.0.bias"]
    time = time / (1.0 + np.exp(-time))
    time = time @ w["time_embedder.mlp.2.weight"].T + w["time_embedder.mlp.2.bias"]
    pe = w["latent_pos_embed.pe"].reshape(c.max_latent_frames, H)
    x = x + time + pe[np.minimum(np.arange(n), c.max_latent_frames - 1)]
    nh, kvh, hd = c.num_attention_heads, c.num_key_value_heads, c.head_dim
    pos = np.arange(length, length + n, dtype=np.float64)
    for li in range(c.num_hidden_layers):
        p = f"model.layers.{li}."
        h = _rms(x, w[p + "nar_input_layernorm.weight"], c.rms_norm_eps)
        q = (h @ w[p + "nar_self_attn.q_proj.weight"].T).reshape(n, nh, hd)
        k = (h @ w[p + "nar_self_attn.k_proj.weight"].T).reshape(n, kvh, hd)
        v = (h @ w[p + "nar_self_attn.v_proj.weight"].T).reshape(n, kvh, hd)
        q = _rope(_rms(q, w[p + "nar_self_attn.q_norm.weight"], c.rms_norm_eps), pos, c)
        k = _rope(_rms(k, w[p + "nar_self_attn.k_norm.weight"], c.rms_norm_eps), pos, c)
        K = np.concatenate([keys[li].reshape(length, kvh, hd), k])
        V = np.concatenate([values[li].reshape(length, kvh, hd), v])
        att = np.empty((n, nh, hd))
        for head in range(nh):
            kh = head // (nh // kvh)
            s = q[:, head] @ K[:, kh].T / math.sqrt(hd)  # every key visible: no mask
            s = np.exp(s - s.max(-1, keepdims=True))
            att[:, head] = (s / s.sum(-1, keepdims=True)) @ V[:, kh]
        x = x + att.reshape(n, nh * hd) @ w[p + "nar_self_attn.o_proj.weight"].T
        h = _rms(x, w[p + "nar_pre_mlp_layernorm.weight"], c.rms_norm_eps)
        g = h @ w[p + "nar_mlp.gate_proj.weight"].T
        u = h @ w[p + "nar_mlp.up_proj.weight"].T
        x = x + (g / (1.0 + np.exp(-g)) * u) @ w[p + "nar_mlp.down_proj.weight"].T
    fin = _rms(x, w["model.norm.weight"], c.rms_norm_eps)
    return (fin @ w["llm2vae.weight"].T + w["llm2vae.bias"])[1:n - 1]


def _bf16(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("prefix,rows,t", [(24, 20, 0.8), (0, 3, 0.25)])
def test_oracle_velocity_matches_numpy_restatement(nar, c1_config, c1_prompt, prefix, rows, t):
    m, w = nar
    cache = m.cache(prefix + rows + 2)
    if prefix:
        m.prefill(c1_prompt[0][:prefix], cache, logits=False)
    kv = [cache.read(li) for li in range(c1_config.num_hidden_layers)]
    state = _bf16(np.random.default_rng(prefix + rows).standard_normal((rows, c1_config.latent_dim)))
    raw_t = math.log(t / (1.0 - t))
    got = m.velocity(state, cache, raw_t)
    want = _velocity(w, c1_config, state.astype(np.float64), [k for k, _ in kv], [v for _, v in kv], prefix, raw_t)
    assert np.isfinite(got).all() and np.array_equal(got, _bf16(got))
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel <= REL_L2, rel
    # the cache is read, not written
    assert cache.length == prefix
    for li, (k, v) in enumerate(kv):
        k2, v2 = cache.read(li)
        assert np.array_equal(k, k2) and np.array_equal(v, v2)
    cache.close()


def test_oracle_velocity_sees_later_latent_rows(nar, c1_config):
    """No causal mask: changing the last latent frame moves the first frame's velocity."""
    m, _ = nar
    cache = m.cache(16)
    s = _bf16(np.random.default_rng(4).standard_normal((6, c1_config.latent_dim)))
    a = m.velocity(s, cache, 0.3)
    s2 = s.copy()
    s2[-1] += 1.0
    b = m.velocity(s2, cache, 0.3)
    assert not np.array_equal(a[0], b[0])
    cache.close()
