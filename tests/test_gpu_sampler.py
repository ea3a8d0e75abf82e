"""Device sampling::choose + MT19937 stream against the oracle: token ids and the
generator state must be bit-identical given identical logits."""
import numpy as np
import pytest

from oracle.oracle import OracleRng
from oracle.oracle import choose as ochoose
from yue2_rs_b200 import Generator, Phase, Sampling, Yue2Error
from yue2_rs_b200 import choose as dchoose

pytestmark = pytest.mark.gpu


def same_state(dev, orc):
    a, na = dev.state()
    b, nb = orc.state()
    return na == nb and (a == b).all()


def run(model, logits, s, hist, step, phase, legacy, seed, reps=3):
    d, o = Generator(model, seed), OracleRng(seed)
    for _ in range(reps):
        a = dchoose(model, logits, s, hist, step, phase, legacy, d)
        b = ochoose(logits, s, hist, step, phase, legacy, o)
        assert a == b
        assert same_state(d, o)
    return a


def bf(x):
    return (np.asarray(x, dtype=np.float32).view(np.uint32) & 0xFFFF0000).view(np.float32)


def test_config1_sampling_bit_exact(c1_device):
    rng = np.random.default_rng(11)
    s = Sampling(1.0, 0.93, 50, 1.0, 50, 0, 512)
    for i in range(40):
        x = bf(rng.standard_normal(84000) * rng.uniform(0.5, 4))
        run(c1_device, x, s, [], i, Phase.VOCAB, False, seed=i)


@pytest.mark.parametrize("kw", [
    dict(temperature=0.7, top_p=0.9, top_k=30, repetition_penalty=1.005, penalty_window=100),
    dict(temperature=1.3, top_p=1.0, top_k=100, repetition_penalty=1.2, penalty_window=50),
    dict(temperature=1.0, top_p=0.95, top_k=1, repetition_penalty=1.2, penalty_window=50),
    dict(temperature=1.0, top_p=0.5, top_k=5000, repetition_penalty=2.0, penalty_window=7),
    dict(temperature=0.0, top_p=0.95, top_k=100, repetition_penalty=1.2, penalty_window=50),
])
@pytest.mark.parametrize("legacy", [False, True])
def test_sampling_configurations(c1_device, kw, legacy):
    rng = np.random.default_rng(5)
    s = Sampling(min_tokens=0, max_tokens=1000, **kw)
    for i in range(6):
        x = bf(rng.standard_normal(84000) * 2)
        hist = rng.integers(0, 84000, size=rng.integers(0, 120)).tolist()
        hist += hist[:10]  # repeated ids
        run(c1_device, x, s, hist, len(hist), Phase.VOCAB, legacy, seed=100 + i)


def test_degenerate_supports_use_the_large_sort(c1_device):
    s = Sampling(1.0, 0.99, 10 ** 9, 1.0, 50, 0, 10)  # top_k beyond the vocabulary keeps every finite id
    x = bf(np.random.default_rng(2).standard_normal(84000))
    run(c1_device, x, s, [], 0, Phase.VOCAB, False, seed=3, reps=2)
    flat = np.zeros(84000, dtype=np.float32)  # all ties: every id survives top-k
    run(c1_device, flat, Sampling(1.0, 0.9, 50, 1.0, 50, 0, 10), [], 0, Phase.VOCAB, False, seed=4, reps=2)
    signed = np.where(np.arange(84000) % 2, np.float32(0.0), np.float32(-0.0)).astype(np.float32)
    run(c1_device, signed, Sampling(0.8, 0.9, 50, 1.0, 50, 0, 10), [], 0, Phase.VOCAB, False, seed=5, reps=2)
    masked = np.full(84000, -np.inf, dtype=np.float32)
    masked[[7, 70000]] = [1.0, 1.0]
    run(c1_device, masked, Sampling(1.0, 0.9, 50, 1.0, 50, 0, 10), [], 0, Phase.VOCAB, False, seed=6, reps=4)


def test_phase_windows_and_stop_gate(c1_device):
    V = 184704
    rng = np.random.default_rng(8)
    x = bf(rng.standard_normal(V))
    x[151852] = 50.0  # MUSIC_END: only eligible from step >= min_tokens
    s = Sampling(1.0, 0.95, 100, 1.2, 50, 3, 100)
    assert run(c1_device, x, s, [151900], 1, Phase.SEMANTIC, False, seed=1) != 151852
    assert run(c1_device, x, s, [151900], 3, Phase.SEMANTIC, False, seed=1) == 151852
    x[151848] = 50.0  # ABC_END
    run(c1_device, x, s, [10, 20], 5, Phase.ABC, True, seed=2)
    with pytest.raises(Yue2Error):
        dchoose(c1_device, x[:84000], s, [], 0, Phase.SEMANTIC, False, Generator(c1_device, 1))


def test_invalid_and_empty(c1_device):
    s = Sampling(1.0, 0.9, 50, 1.0, 50, 0, 10)
    x = np.zeros(84000, dtype=np.float32)
    x[5] = np.nan
    with pytest.raises(Yue2Error, match="invalid logits"):
        dchoose(c1_device, x, s, [], 0, Phase.VOCAB, False, Generator(c1_device, 1))
    with pytest.raises(Yue2Error, match="Empty"):
        dchoose(c1_device, np.full(84000, -np.inf, dtype=np.float32), s, [], 0, Phase.VOCAB, False,
                Generator(c1_device, 1))
