"""detmath.h (shared by the device sampler and the oracle) against libm."""
import math

import numpy as np

from oracle.oracle import lib


def test_expf_is_correctly_rounded():
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-104, 89, 100000), rng.uniform(-1, 1, 20000), [0.0, -0.0, 1.0, -1.0,
                         88.72, 88.73, -87.3, -103.9, -104.0, -110.0, -200.0, 100.0]]).astype(np.float32)
    L = lib()
    bad = 0
    for x in xs:
        got = L.orc_det_expf(float(x))
        try:
            want = float(np.float32(math.exp(float(x))))
        except OverflowError:
            want = math.inf
        if not (got == want):
            bad += 1
    assert bad == 0


def test_expf_specials():
    L = lib()
    assert math.isnan(L.orc_det_expf(float("nan")))
    assert L.orc_det_expf(float("-inf")) == 0.0
    assert L.orc_det_expf(float("inf")) == math.inf


def test_log1p_matches_libm():
    rng = np.random.default_rng(1)
    L = lib()
    us = np.concatenate([rng.random(100000), [0.0, 1e-300, 2.0 ** -53, 0.5, 1 - 2.0 ** -53]])
    for u in us:
        got, want = L.orc_det_log1p(-float(u)), math.log1p(-float(u))
        assert abs(got - want) <= 2 * abs(math.ulp(want)) + 1e-300
        # the sampler only uses the float cast of -log1p(-u)
        assert np.float32(-got) == np.float32(-want)
    assert math.copysign(1.0, L.orc_det_log1p(-0.0)) == -1.0
    assert L.orc_det_log1p(-1.0) == -math.inf


def test_round_bf16_and_powi():
    L = lib()
    # ties to even, NaN quieted with the sign kept, overflow to inf (tensor.rs:645-652)
    assert L.orc_round_bf16(1.0 + 2 ** -8) == 1.0
    assert L.orc_round_bf16(1.0 + 3 * 2 ** -8) == 1.0 + 2 ** -6
    assert L.orc_round_bf16(3.4028234663852886e38) == math.inf  # FLT_MAX rounds up past the largest bf16
    assert L.orc_round_bf16(3.3895313892515355e38) == 3.3895313892515355e38
    nan = np.array([0xFFC00001], dtype=np.uint32).view(np.float32)[0]
    r = np.array([L.orc_round_bf16(float(nan))], dtype=np.float32).view(np.uint32)[0]
    assert r == 0xFFC00000
    for a in (1.2, 1.005, 0.9, 2.5):
        for n in range(1, 60):
            want = np.float32(1.0)
            base, e = np.float32(a), n
            while True:  # the same binary exponentiation, in numpy float32
                if e & 1:
                    want = np.float32(want * base)
                e //= 2
                if e == 0:
                    break
                base = np.float32(base * base)
            assert L.orc_powi(np.float32(a), n) == want
