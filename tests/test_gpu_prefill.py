"""GEMM prefill (prompts of >= 64 ids as bf16 tensor-core GEMMs over chunks of consecutive
positions, Model::prefill_phase, src/model.rs:508-522).

  * against the oracle within the north_star tolerance, with a chunk size small enough that
    later chunks attend to K/V written by earlier ones;
  * against the GEMV prefill (YUE2_CUDA_PREFILL=gemv) on the unit-gain model: same math,
    other f32 summation order;
  * the tensor-core causal attention against the per-row decode attention kernel
    (YUE2_CUDA_PREFILL_ATTN=rows) over a 1,000-id prompt in chunks of 250 positions;
  * appending to a non-empty cache, and run-to-run determinism (bit-exact logits and K/V).
"""
import os

import numpy as np
import pytest

from oracle import oracle as orc
from yue2_rs_b200 import Model

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def _open(path, **env):
    old = {k: os.environ.get(k) for k in env}
    os.environ.update({k: str(v) for k, v in env.items()})
    try:
        return Model.open(path)
    finally:
        for k, v in old.items():
            if v is None:
                del os.environ[k]
            else:
                os.environ[k] = v


@pytest.fixture(scope="module")
def chunked(c1_dir):
    m = _open(c1_dir, YUE2_CUDA_PREFILL_CHUNK=96)
    yield m
    m.close()


@pytest.fixture(scope="module")
def rows_u(c1u_dir):
    m = _open(c1u_dir, YUE2_CUDA_PREFILL_ATTN="rows", YUE2_CUDA_PREFILL_CHUNK=300)
    yield m
    m.close()


@pytest.fixture(scope="module")
def chunk300_u(c1u_dir):
    m = _open(c1u_dir, YUE2_CUDA_PREFILL_CHUNK=300)
    yield m
    m.close()


@pytest.fixture(scope="module")
def gemv_u(c1u_dir):
    m = _open(c1u_dir, YUE2_CUDA_PREFILL="gemv")
    yield m
    m.close()


def _decode(model, prompt, teacher, split=None):
    c = model.new_cache(len(prompt) + len(teacher))
    if split:
        model.forward(prompt[:split], c)
        first = model.forward(prompt[split:], c)
    else:
        first = model.forward(prompt, c)
    return np.array([first] + [model.forward([t], c) for t in teacher]), c


def test_chunked_gemm_prefill_matches_oracle(chunked, c1_oracle, c1_prompt):
    prompt, teacher = c1_prompt
    teacher = teacher[:16]
    dev, dc = _decode(chunked, prompt, teacher)  # 256 ids: chunks of 86, 85, 85
    c = c1_oracle.cache(len(prompt) + len(teacher))
    ref = np.array([c1_oracle.prefill(prompt, c)] + [c1_oracle.forward([t], c) for t in teacher])
    for step in range(len(dev)):
        d = np.abs(dev[step].astype(np.float64) - ref[step])
        assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, (step, d.max(), d.mean())
    to_f = lambda b: (b.astype(np.uint32) << 16).view(np.float32)
    for layer in range(c1_oracle.config.num_hidden_layers):
        kd, vd = dc.read(layer, 0, dc.length)
        ko, vo = c.read(layer)
        assert np.mean(to_f(kd) == ko) > 0.9 and np.mean(to_f(vd) == vo) > 0.9


def test_gemm_prefill_matches_gemv_prefill(c1u_device, gemv_u, c1_prompt):
    prompt, teacher = c1_prompt
    a, ca = _decode(c1u_device, prompt, teacher[:8])
    b, cb = _decode(gemv_u, prompt, teacher[:8])
    assert np.isfinite(a).all()
    # the same bf16 roundings in another f32 summation order: most logits within an ulp
    assert np.abs(a - b).max() <= 0.08
    assert np.abs(a - b).mean() <= 1e-2
    assert (a.argmax(-1) == b.argmax(-1)).mean() >= 0.9
    # layer 0's K/V see only the projection's summation order (rare bf16 flips); deeper
    # layers also inherit the ulp differences of the unit-gain residual stream
    to_f = lambda x: (x.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    for layer in range(2):
        ka, va = ca.read(layer, 0, len(prompt))
        kb, vb = cb.read(layer, 0, len(prompt))
        if layer == 0:
            assert np.mean(ka == kb) > 0.9 and np.mean(va == vb) > 0.9
        for x, y in ((ka, kb), (va, vb)):
            x, y = to_f(x), to_f(y)
            assert np.linalg.norm(x - y) <= 2e-2 * np.linalg.norm(y)


def test_gemm_prefill_appends_to_a_cache(c1u_device, gemv_u, c1_prompt):
    prompt, teacher = c1_prompt
    # 100 ids, then 156 more starting at position 100 (both GEMM prefills)
    a, _ = _decode(c1u_device, prompt, teacher[:4], split=100)
    b, _ = _decode(gemv_u, prompt, teacher[:4], split=100)
    assert np.abs(a - b).max() <= 0.08 and np.abs(a - b).mean() <= 1e-2
    assert (a.argmax(-1) == b.argmax(-1)).mean() >= 0.9


def test_gemm_prefill_is_deterministic(c1u_device, c1_prompt):
    prompt = c1_prompt[0]
    a, ca = _decode(c1u_device, prompt, [])
    b, cb = _decode(c1u_device, prompt, [])
    assert np.array_equal(a, b)
    for layer in range(2):
        ka, va = ca.read(layer, 0, len(prompt))
        kb, vb = cb.read(layer, 0, len(prompt))
        assert np.array_equal(ka, kb) and np.array_equal(va, vb)


def test_tensor_core_attention_matches_row_attention(chunk300_u, rows_u, c1_config):
    rng = np.random.default_rng(11)
    prompt = rng.integers(0, c1_config.vocab_size, 1000).tolist()
    teacher = rng.integers(0, c1_config.vocab_size, 4).tolist()
    a, ca = _decode(chunk300_u, prompt, teacher)
    b, cb = _decode(rows_u, prompt, teacher)
    assert np.isfinite(a).all()
    assert np.abs(a - b).max() <= 0.08 and np.abs(a - b).mean() <= 1e-2
    assert (a.argmax(-1) == b.argmax(-1)).mean() >= 0.9
    # layer 0's K/V do not depend on attention; layer 1's inherit its summation order
    ka, va = ca.read(0, 0, len(prompt))
    kb, vb = cb.read(0, 0, len(prompt))
    assert np.array_equal(ka, kb) and np.array_equal(va, vb)
    to_f = lambda x: (x.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    ka, va = ca.read(1, 0, len(prompt))
    kb, vb = cb.read(1, 0, len(prompt))
    for x, y in ((ka, kb), (va, vb)):
        assert np.linalg.norm(to_f(x) - to_f(y)) <= 2e-2 * np.linalg.norm(to_f(y))
