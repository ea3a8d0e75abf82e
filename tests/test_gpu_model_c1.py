"""teacher-forced per-step logits of the CUDA path against the
oracle's restatement of the reference decode path (tolerance 2e-2 max-abs, 1e-3 mean-abs)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 1e-3


def compare(got, want, what):
    d = np.abs(got.astype(np.float64) - want.astype(np.float64))
    assert np.isfinite(got).all(), what
    assert d.max() <= MAX_ABS and d.mean() <= MEAN_ABS, f"{what}: max {d.max():.3g} mean {d.mean():.3g}"
    return d.max(), d.mean()


def test_teacher_forced_logits_config0(c1_device, c1_oracle, c1_prompt):
    prompt, teacher = c1_prompt
    cap = len(prompt) + len(teacher)
    dc = c1_device.new_cache(cap)
    oc = c1_oracle.cache(cap)
    compare(c1_device.forward(prompt, dc), c1_oracle.prefill(prompt, oc), "prefill")
    worst = []
    for step, tok in enumerate(teacher):
        worst.append(compare(c1_device.forward([tok], dc), c1_oracle.forward([tok], oc), f"step {step}"))
    assert dc.length == oc.length == cap
    # the KV caches agree except for rare bf16 rounding flips
    for layer in range(c1_oracle.config.num_hidden_layers):
        kd, vd = dc.read(layer, 0, cap)
        ko, vo = oc.read(layer)
        to_f = lambda b: (b.astype(np.uint32) << 16).view(np.float32)
        assert np.mean(to_f(kd) == ko) > 0.99 and np.mean(to_f(vd) == vo) > 0.99


def test_batched_rows_equal_single_rows(c1_device, c1_prompt):
    """Rows in one weight pass do not interact: R=3 gives the R=1 logits bit for bit."""
    prompt, teacher = c1_prompt
    caches = [c1_device.new_cache(64) for _ in range(3)]
    singles = [c1_device.new_cache(64) for _ in range(3)]
    for i in range(3):
        c1_device.forward(prompt[i * 5: i * 5 + 7], caches[i])
        c1_device.forward(prompt[i * 5: i * 5 + 7], singles[i])
    rows = c1_device.forward_rows(caches, teacher[:3])
    for i in range(3):
        one = c1_device.forward([teacher[i]], singles[i])
        assert (rows[i].view(np.uint32) == one.view(np.uint32)).all()


def test_capacity_and_token_errors(c1_device):
    from yue2_rs_b200 import Yue2Error
    c = c1_device.new_cache(2)
    c1_device.forward([1, 2], c)
    with pytest.raises(Yue2Error, match="exceeds cache"):
        c1_device.forward([3], c)
    with pytest.raises(Yue2Error, match="outside model vocabulary"):
        c1_device.forward([c1_device.config.vocab_size], c1_device.new_cache(4))
    with pytest.raises(Yue2Error, match="native music protocol"):
        from yue2_rs_b200 import Phase
        c1_device.forward_phase([1], c1_device.new_cache(4), Phase.SEMANTIC)
