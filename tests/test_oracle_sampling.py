"""The oracle's sampling::choose / CFG mix (src/sampling.rs:103-266) on hand-built logits."""
import numpy as np
import pytest

from oracle.oracle import OracleError, OracleRng, cfg_mix, choose
from refmath import round_bf16_np
from yue2_rs_b200.protocol import Phase, Sampling

V = 4096


def greedy():
    return Sampling(temperature=0.0, top_p=1.0, top_k=10, repetition_penalty=1.0, penalty_window=50, min_tokens=0,
                    max_tokens=10)


def test_greedy_ties_take_lowest_id_and_positive_zero_wins():
    x = np.full(V, -5.0, dtype=np.float32)
    x[[10, 20, 30]] = 2.0
    assert choose(x, greedy(), [], 0, Phase.VOCAB, False, OracleRng(1)) == 10
    x = np.full(V, -np.inf, dtype=np.float32)
    x[5], x[3] = 0.0, -0.0
    assert choose(x, greedy(), [], 0, Phase.VOCAB, False, OracleRng(1)) == 5


def test_greedy_draws_nothing_sampled_draws_two_words_per_id():
    x = np.random.default_rng(0).standard_normal(V).astype(np.float32)
    g = OracleRng(3)
    choose(x, greedy(), [], 0, Phase.VOCAB, False, g)
    st, nxt = g.state()
    assert nxt == 624  # untouched
    s = Sampling(1.0, 0.9, 50, 1.0, 50, 0, 10)
    choose(x, s, [], 0, Phase.VOCAB, False, g)
    ref = OracleRng(3)
    ref.discard(2 * V)
    assert all((a == b).all() if hasattr(a, "all") else a == b for a, b in zip(g.state(), ref.state()))


def test_repetition_penalty_divides_positive_and_multiplies_negative():
    x = np.full(V, -9.0, dtype=np.float32)
    x[5], x[7] = 3.0, 2.0
    s = greedy()
    s.repetition_penalty = 2.0
    assert choose(x, s, [5], 0, Phase.VOCAB, False, OracleRng(1)) == 7  # 3/2 < 2
    assert choose(x, s, [5, 9, 9], 0, Phase.VOCAB, False, OracleRng(1)) == 7
    x = np.full(V, -9.0, dtype=np.float32)
    x[5], x[7] = -1.0, -1.5
    assert choose(x, s, [5], 0, Phase.VOCAB, False, OracleRng(1)) == 7  # -1*2 < -1.5
    # only the last penalty_window ids count
    s.penalty_window = 1
    x[5], x[7] = 3.0, 2.0
    assert choose(x, s, [5, 9], 0, Phase.VOCAB, False, OracleRng(1)) == 5


def test_invalid_and_empty_distributions():
    s = Sampling(1.0, 0.9, 50, 1.0, 50, 0, 10)
    x = np.zeros(V, dtype=np.float32)
    x[3] = np.nan
    with pytest.raises(OracleError, match="invalid logits"):
        choose(x, s, [], 0, Phase.VOCAB, False, OracleRng(1))
    x[3] = np.inf
    with pytest.raises(OracleError, match="invalid logits"):
        choose(x, s, [], 0, Phase.VOCAB, False, OracleRng(1))
    with pytest.raises(OracleError, match="Empty"):
        choose(np.full(V, -np.inf, dtype=np.float32), s, [], 0, Phase.VOCAB, False, OracleRng(1))
    with pytest.raises(OracleError, match="native music protocol"):
        choose(np.zeros(V, dtype=np.float32), s, [], 0, Phase.SEMANTIC, False, OracleRng(1))


def test_exponential_race_draws_the_softmax_distribution():
    logits = np.log(np.array([0.1, 0.2, 0.3, 0.4], dtype=np.float64)).astype(np.float32)
    s = Sampling(1.0, 1.0, 4, 1.0, 50, 0, 10)
    g = OracleRng(2024)
    counts = np.zeros(4)
    n = 40000
    for _ in range(n):
        counts[choose(logits, s, [], 0, Phase.VOCAB, False, g)] += 1
    assert np.allclose(counts / n, [0.1, 0.2, 0.3, 0.4], atol=0.01)


def test_top_k_and_top_p_restrict_support():
    logits = np.linspace(0, 3, 16).astype(np.float32)
    g = OracleRng(9)
    s = Sampling(1.0, 1.0, 3, 1.0, 50, 0, 10)
    assert {choose(logits, s, [], 0, Phase.VOCAB, False, g) for _ in range(300)} <= {13, 14, 15}
    s = Sampling(1.0, 1e-6, 16, 1.0, 50, 0, 10)  # top_p keeps only the protected first id
    assert {choose(logits, s, [], 0, Phase.VOCAB, False, g) for _ in range(50)} == {15}
    s.top_p = 1e-6
    assert {choose(logits, s, [], 0, Phase.VOCAB, True, g) for _ in range(200)} <= {13, 14, 15}  # legacy: 3


def test_ties_at_the_top_k_threshold_all_survive():
    x = np.full(64, -3.0, dtype=np.float32)
    x[[4, 9, 17, 33]] = 1.0
    s = Sampling(1.0, 1.0, 2, 1.0, 50, 0, 10)
    g = OracleRng(5)
    assert {choose(x, s, [], 0, Phase.VOCAB, False, g) for _ in range(400)} == {4, 9, 17, 33}


def test_cfg_mix_formula():
    rng = np.random.default_rng(4)
    c = round_bf16_np(rng.standard_normal(5000).astype(np.float32) * 3)
    u = round_bf16_np(rng.standard_normal(5000).astype(np.float32) * 3)
    s = np.float32(1.5)
    want = round_bf16_np(u + round_bf16_np(s * round_bf16_np(c - u)))
    assert (cfg_mix(c, u, 1.5).view(np.uint32) == want.view(np.uint32)).all()
