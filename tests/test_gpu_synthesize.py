"""Model::synthesize (src/model.rs:699-776) on the device against the oracle, on the small
real-vocabulary model (head_dim 64, a 160-position context, so a 150-frame song runs as
three chunks of 63 + 63 + 24 frames):

  * the latents' displacement from the starting noise (what the flow ODE adds) within the
    velocity tolerance of the oracle's, after 2 and 3 midpoint steps;
  * the velocity itself at head_dim 64 after a real-vocabulary prefill;
  * run-to-run determinism, and the reference's argument errors.
"""
import numpy as np
import pytest

from oracle import oracle as orc
from yue2_rs_b200 import Model, _lib, checkpoint, synth

pytestmark = pytest.mark.gpu

REL_L2 = 3e-2  # two velocity evaluations per step, each within 2e-2 of the oracle's


def _bf16(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32).view(np.float32)


@pytest.fixture(scope="module")
def dev(nar_tiny_dir):
    m = Model.open(nar_tiny_dir, nar=True)
    yield m
    m.close()


@pytest.fixture(scope="module")
def ora(nar_tiny_dir):
    m = orc.OracleModel.from_tensors(synth.config_nar_tiny(), checkpoint.tensors(nar_tiny_dir), nar=True)
    yield m
    m.close()


def _song(seed):
    rng = np.random.default_rng(seed)
    return rng.integers(0, 184704, 30).tolist(), rng.integers(0, 32768, 150).tolist()


@pytest.mark.parametrize("steps", [2, 3])
def test_synthesize_matches_oracle(dev, ora, steps):
    prefix, codec = _song(steps)
    a = dev.synthesize(prefix, codec, seed=7, steps=steps)
    b = ora.synthesize(prefix, codec, seed=7, steps=steps)
    z = _bf16(orc.normal_tensor(7, len(codec), 64))
    assert a.shape == b.shape == (150, 64) and np.isfinite(a).all()
    assert np.array_equal(a, _bf16(a))
    da, db = a - z, b - z
    rel = np.linalg.norm(da - db) / np.linalg.norm(db)
    assert rel <= REL_L2, rel
    for lo, hi in ((0, 63), (63, 126), (126, 150)):  # every chunk moved, and alike
        assert np.linalg.norm(db[lo:hi]) > 0
        assert np.linalg.norm(da[lo:hi] - db[lo:hi]) <= REL_L2 * np.linalg.norm(db[lo:hi])
    assert np.array_equal(a, dev.synthesize(prefix, codec, seed=7, steps=steps))


def test_velocity_head_dim_64_after_real_vocab_prefill(dev, ora):
    prefix, codec = _song(11)
    ids = prefix + [151853 + t for t in codec[:40]] + [151852]
    rows = 40
    dc, _ = dev.prefill(ids, len(ids) + rows + 2, logits=False)
    oc = ora.cache(len(ids))
    ora.prefill(ids, oc, logits=False)
    st = _bf16(np.random.default_rng(5).standard_normal((rows, 64)))
    a, b = dev.velocity(st, dc, 1.5), ora.velocity(st, oc, 1.5)
    assert np.linalg.norm(a - b) <= 2e-2 * np.linalg.norm(b)
    dc.close()


def test_synthesize_errors(dev, c1_device):
    with pytest.raises(_lib.Yue2Error):
        dev.synthesize([1, 2], [32768], seed=1, steps=1)  # codec id out of range
    with pytest.raises(_lib.Yue2Error):
        dev.synthesize([1, 2], [], seed=1, steps=1)
    with pytest.raises(_lib.Yue2Error):
        dev.synthesize([1, 2], [5], seed=1, steps=0)
    with pytest.raises(_lib.Yue2Error):
        dev.synthesize(list(range(156)), [5], seed=1, steps=1)  # no acoustic context left
    with pytest.raises(_lib.Yue2Error):
        c1_device.synthesize([1, 2], [5], seed=1, steps=1)  # NAR tensors not loaded
