"""The acoustic stage's host parts, on CPU:

  * Generator::normal_tensor (src/sampling.rs:63-78): the library's host noise is bit-exact
    against the oracle's, and both follow the reference's layout (uniform_f32 draws from
    the MT19937 stream that the std::mt19937 known answers pin, then Box-Muller pairs i and
    i + 8 of every 16-element block), checked against a float64 numpy restatement;
  * Model::synthesize (src/model.rs:699-776) in the oracle against a Python restatement of
    its loop over the oracle's own prefill and velocity: the chunk sizes, the ids of each
    chunk, the noise slices, the midpoint updates and their roundings, bit-exact;
  * the reference's argument errors.
"""
import math

import numpy as np
import pytest

from oracle import oracle as orc
from yue2_rs_b200 import _lib, checkpoint, synth
from yue2_rs_b200.model import noise

CODEC_OFFSET, MUSIC_END = 151853, 151852


def _bf16(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)


@pytest.mark.parametrize("seed,rows", [(831001, 100), (0, 1), (2**40 + 7, 333), (12345, 640)])
def test_library_noise_is_the_oracle_noise(seed, rows):
    a, b = noise(seed, rows, 64), orc.normal_tensor(seed, rows, 64)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_noise_layout_against_numpy():
    seed, rows = 77, 40
    rng = orc.OracleRng(seed)
    u = np.array([rng.uniform_f32() for _ in range(rows * 64)], dtype=np.float32).reshape(-1, 16)
    r = np.sqrt(-2.0 * np.log(1.0 - u[:, :8].astype(np.float64)))
    th = (2.0 * math.pi * u[:, 8:].astype(np.float64)).astype(np.float32).astype(np.float64)
    want = np.concatenate([r * np.cos(th), r * np.sin(th)], 1).reshape(rows, 64)
    got = orc.normal_tensor(seed, rows, 64)
    assert np.abs(got - want).max() <= 1e-5 * max(1.0, np.abs(want).max())
    assert abs(got.mean()) < 0.1 and abs(got.std() - 1.0) < 0.1


def test_noise_needs_blocks_of_16():
    with pytest.raises(_lib.Yue2Error):
        noise(1, 1, 8)


@pytest.fixture(scope="module")
def tiny(nar_tiny_dir):
    c = synth.config_nar_tiny()
    m = orc.OracleModel.from_tensors(c, checkpoint.tensors(nar_tiny_dir), nar=True)
    yield m, c
    m.close()


def _logit(t):
    with np.errstate(divide="ignore"):
        v = np.log(np.float64(t) / (1.0 - np.float64(t)))
    return float(min(20.0, max(-20.0, v)))


def _synthesize(m, c, prefix, codec, seed, steps):
    """model.rs:699-776 over the oracle's prefill and velocity."""
    capacity = min(24576, c.max_position_embeddings)
    size = (capacity - (len(prefix) + 3)) // 2
    z = orc.normal_tensor(seed, len(codec), 64)
    dt = np.float32(1.0) / np.float32(steps)
    out = []
    for start in range(0, len(codec), size):
        end = min(start + size, len(codec))
        ids = list(prefix) + [t + CODEC_OFFSET for t in codec[start:end]] + [MUSIC_END]
        cache = m.cache(len(ids))
        m.prefill(ids, cache, logits=False)
        state = _bf16(z[start:end])
        for step in range(steps):
            t = 1.0 - step / steps
            first = m.velocity(state, cache, _logit(t))
            mid = _bf16(state - _bf16(first * (dt / np.float32(2.0))))
            v = m.velocity(mid, cache, _logit(t - 0.5 / steps))
            state = _bf16(state - _bf16(v * dt))
        cache.close()
        out.append(state)
    return np.concatenate(out)


def test_oracle_synthesize_is_the_reference_loop(tiny):
    m, c = tiny
    rng = np.random.default_rng(3)
    prefix = rng.integers(0, c.vocab_size, 30).tolist()
    codec = rng.integers(0, 32768, 150).tolist()  # chunks of (160 - 33) // 2 = 63: 63 + 63 + 24
    got = m.synthesize(prefix, codec, seed=99, steps=2)
    want = _synthesize(m, c, prefix, codec, 99, 2)
    assert got.shape == (150, 64) and np.isfinite(got).all()
    assert np.array_equal(got, want)
    assert not np.array_equal(got, _bf16(orc.normal_tensor(99, 150, 64)))  # the ODE moved the noise


@pytest.mark.parametrize("frames,steps", [(126, 1), (1, 2), (64, 3)])
def test_oracle_synthesize_chunk_edges(tiny, frames, steps):
    """Two full chunks of 63 (no remainder), a one-frame song, and one chunk plus one frame."""
    m, c = tiny
    rng = np.random.default_rng(frames)
    prefix = rng.integers(0, c.vocab_size, 30).tolist()
    codec = rng.integers(0, 32768, frames).tolist()
    got = m.synthesize(prefix, codec, seed=frames + 1, steps=steps)
    assert got.shape == (frames, 64)
    assert np.array_equal(got, _synthesize(m, c, prefix, codec, frames + 1, steps))


def test_oracle_synthesize_errors(tiny):
    m, c = tiny
    with pytest.raises(orc.OracleError):
        m.synthesize([1, 2], [32768], seed=1, steps=1)  # codec id out of range
    with pytest.raises(orc.OracleError):
        m.synthesize([1, 2], [], seed=1, steps=1)
    with pytest.raises(orc.OracleError):
        m.synthesize([1, 2], [5], seed=1, steps=0)
    with pytest.raises(orc.OracleError):
        m.synthesize(list(range(156)), [5], seed=1, steps=1)  # (160 - 159) // 2 == 0
