"""NAR flow-matching velocity (Model::velocity, src/model.rs:611-697, nar_cond_end 0) on the
device against the oracle, on the unit-gain reduced model with its NAR tensors:

  * after a GEMM-prefilled prompt, for latent blocks shorter than, equal to and longer than
    max_latent_frames (the position table's last row repeats), for a single frame, and for
    1,500 frames (past the 1,024-row prefill chunk: one pass of every layer over all rows);
  * on an empty cache (the latent rows attend only to one another);
  * the cache is left as it was: same length, and the next AR step's logits are bit-exact
    against a twin cache that never ran velocity;
  * argument errors (rows 0, capacity, NAR tensors not loaded).
"""
import math

import numpy as np
import pytest

from oracle import oracle as orc
from yue2_rs_b200 import Model, _lib, checkpoint

pytestmark = pytest.mark.gpu

# the latent outputs are bf16 roundings of f32 sums taken in another order, through the
# same layers as the prefill: the prefill tolerance, relative to the output scale
REL_L2, REL_MAX = 2e-2, 4e-2


def _bf16(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def _logit(t):
    return math.log(t / (1.0 - t))


@pytest.fixture(scope="module")
def nar_device(c1u_dir):
    m = Model.open(c1u_dir, nar=True)
    yield m
    m.close()


@pytest.fixture(scope="module")
def nar_oracle(c1u_dir, c1_config):
    m = orc.OracleModel.from_tensors(c1_config, checkpoint.tensors(c1u_dir), nar=True)
    yield m
    m.close()


def _state(rows, latent, seed):
    return _bf16(np.random.default_rng(seed).standard_normal((rows, latent)))


def _compare(a, b):
    assert a.shape == b.shape and np.isfinite(a).all()
    assert np.array_equal(a, _bf16(a))  # bf16-valued, as Linear::finish leaves them
    rel = np.linalg.norm(a - b) / np.linalg.norm(b)
    mx = np.abs(a - b).max() / np.abs(b).max()
    assert rel <= REL_L2 and mx <= REL_MAX, (rel, mx)
    return rel, mx


@pytest.mark.parametrize("rows,t,seed", [(14, 0.9, 1), (30, 0.3, 2), (1, 0.55, 3), (1500, 0.7, 4)])
def test_velocity_matches_oracle_after_prefill(nar_device, nar_oracle, c1_prompt, c1_config, rows, t, seed):
    prompt = c1_prompt[0][:40]
    cap = len(prompt) + rows + 2
    dc, _ = nar_device.prefill(prompt, cap, logits=False)
    oc = nar_oracle.cache(cap)
    nar_oracle.prefill(prompt, oc, logits=False)
    state = _state(rows, c1_config.latent_dim, seed)
    a = nar_device.velocity(state, dc, _logit(t))
    b = nar_oracle.velocity(state, oc, _logit(t))
    _compare(a, b)
    dc.close()


def test_velocity_on_an_empty_cache(nar_device, nar_oracle, c1_config):
    state = _state(5, c1_config.latent_dim, 7)
    dc = nar_device.new_cache(16)
    oc = nar_oracle.cache(16)
    _compare(nar_device.velocity(state, dc, _logit(0.6)), nar_oracle.velocity(state, oc, _logit(0.6)))
    dc.close()


def test_velocity_leaves_the_cache_unchanged(nar_device, c1_prompt, c1_config):
    prompt, teacher = c1_prompt[0][:64], c1_prompt[1]
    a, _ = nar_device.prefill(prompt, 128, logits=False)
    b, _ = nar_device.prefill(prompt, 128, logits=False)
    v1 = nar_device.velocity(_state(20, c1_config.latent_dim, 9), a, _logit(0.8))
    assert a.length == len(prompt)
    la = nar_device.forward([teacher[0]], a)
    lb = nar_device.forward([teacher[0]], b)
    assert np.array_equal(la, lb)
    # and the same call again (positions now past the new length) is deterministic
    c, _ = nar_device.prefill(prompt, 128, logits=False)
    nar_device.forward([teacher[0]], c)
    v2 = nar_device.velocity(_state(20, c1_config.latent_dim, 9), c, _logit(0.8))
    v3 = nar_device.velocity(_state(20, c1_config.latent_dim, 9), a, _logit(0.8))
    assert np.array_equal(v2, v3)
    assert v1.shape == v2.shape
    for x in (a, b, c):
        x.close()


def test_velocity_argument_errors(nar_device, c1_device, c1_config):
    L = c1_config.latent_dim
    cache = nar_device.new_cache(8)
    with pytest.raises(_lib.Yue2Error):
        nar_device.velocity(np.zeros((7, L), np.float32), cache, 0.0)  # 7 + 2 > capacity 8
    with pytest.raises(_lib.Yue2Error):
        nar_device.velocity(np.zeros((0, L), np.float32), cache, 0.0)
    cache.close()
    other = c1_device.new_cache(8)
    with pytest.raises(_lib.Yue2Error):
        c1_device.velocity(np.zeros((2, L), np.float32), other, 0.0)  # NAR tensors not loaded
    other.close()
