"""The tcgen05 chunk attention (the default for head_dim 128) against the oracle and
against the mma.sync chunk attention (YUE2_CUDA_PREFILL_ATTN=sync), on the unit-gain
reduced model:

  * causal: a GEMM prefill in chunks of 300 positions (later chunks attend to earlier
    chunks' K/V, partial row tiles) within the prefill tolerance of the oracle;
  * non-causal: NAR velocity over 1,500 latent rows (12 row tiles) after a prefill, within
    the velocity tolerance of the oracle;
  * both paths agree with the mma.sync kernel to f32 summation order.
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from yue2_rs_b200 import Model, checkpoint

pytestmark = pytest.mark.gpu

C1U_MAX, C1U_MEAN = 0.08, 1e-2  # logits of the unit-gain model (as in the prefill tests)


def _open(path, **env):
    old = {k: os.environ.get(k) for k in env}
    os.environ.update({k: str(v) for k, v in env.items()})
    try:
        return Model.open(path, nar=True)
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


def _bf16(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def tc5(c1u_dir):
    m = _open(c1u_dir, YUE2_CUDA_PREFILL_ATTN="tc", YUE2_CUDA_PREFILL_CHUNK=300)
    yield m
    m.close()


@pytest.fixture(scope="module")
def sync(c1u_dir):
    m = _open(c1u_dir, YUE2_CUDA_PREFILL_ATTN="sync", YUE2_CUDA_PREFILL_CHUNK=300)
    yield m
    m.close()


@pytest.fixture(scope="module")
def ora(c1u_dir, c1_config):
    m = orc.OracleModel.from_tensors(c1_config, checkpoint.tensors(c1u_dir), nar=True)
    yield m
    m.close()


def test_causal_prefill_matches_oracle(tc5, sync, ora, c1_config):
    rng = np.random.default_rng(21)
    prompt = rng.integers(0, c1_config.vocab_size, 700).tolist()
    c, a = tc5.prefill(prompt, 720)
    c2, a2 = sync.prefill(prompt, 720)
    oc = ora.cache(720)
    b = ora.prefill(prompt, oc)
    assert np.isfinite(a).all()
    d = np.abs(a.astype(np.float64) - b)
    d2 = np.abs(a2.astype(np.float64) - b)
    # the unit-gain model's logit tolerance, and no further from the oracle than mma.sync
    assert d.max() <= C1U_MAX and d.mean() <= C1U_MEAN, (d.max(), d.mean())
    assert d.mean() <= 1.25 * d2.mean() + 1e-4, (d.mean(), d2.mean())
    assert (a.argmax() == b.argmax())
    c.close()
    c2.close()


def test_non_causal_velocity_matches_oracle(tc5, sync, ora, c1_prompt, c1_config):
    prompt = c1_prompt[0][:40]
    rows = 1500
    st = _bf16(np.random.default_rng(8).standard_normal((rows, c1_config.latent_dim)))
    dc, _ = tc5.prefill(prompt, len(prompt) + rows + 2, logits=False)
    sc, _ = sync.prefill(prompt, len(prompt) + rows + 2, logits=False)
    oc = ora.cache(len(prompt) + rows + 2)
    ora.prefill(prompt, oc, logits=False)
    a = tc5.velocity(st, dc, 0.4)
    c = sync.velocity(st, sc, 0.4)
    b = ora.velocity(st, oc, 0.4)
    assert np.isfinite(a).all()
    rel = np.linalg.norm(a - b) / np.linalg.norm(b)
    rel2 = np.linalg.norm(c - b) / np.linalg.norm(b)
    mx = np.abs(a - b).max() / np.abs(b).max()
    assert rel <= 2e-2 and mx <= 4e-2, (rel, mx)
    assert rel <= 1.25 * rel2 + 1e-4, (rel, rel2)
    dc.close()
    sc.close()
